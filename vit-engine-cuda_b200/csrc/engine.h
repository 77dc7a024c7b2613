// Internal host-side interfaces between the translation units of libvitb200.so.
// Not part of the C ABI (that is include/vitb200.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace vitb200 {

// Row/column mapping of a GEMM epilogue.
enum EpiMode : int {
  kModePlain = 0,  // out row = m
  kModePatch = 1,  // out row = (m / P) * T + 1 + m % P, adds pos[(1 + m % P)][n]
  kModeSplit3 = 2, // column n goes to plane n / e_split, column n % e_split
};

struct GemmEpilogue {
  const float* bias = nullptr;      // [N] or null
  const float* residual = nullptr;  // residual[row*ldr + n] (may alias out)
  int64_t ldr = 0;
  float* out = nullptr;             // fp32 result (row stride ldo) or null
  int64_t ldo = 0;
  float* out_pair = nullptr;        // TF32 pair of the result or null
  int64_t ldp = 0;                  // pair row stride
  int64_t pair_plane = 0;           // elements between the hi and lo planes
  int gelu = 0;                     // apply exact GELU after the bias
  int mode = kModePlain;
  int P = 0, T = 0;                 // kModePatch
  const float* pos = nullptr;       // kModePatch: pos[T][N]
  int e_split = 0;                  // kModeSplit3
  int64_t split_plane = 0;          // kModeSplit3: elements between planes
};

struct GemmProblem {
  const float* a_pair = nullptr;  // [2][M][Kp]
  const float* b_pair = nullptr;  // [2][N][Kp]
  int64_t M = 0;
  int N = 0;
  int Kp = 0;                     // % 4 == 0
  GemmEpilogue epi;
};

// Launches the TF32x3 tcgen05 GEMM; returns a vitb200 status code.
int gemm_pairs_launch(const GemmProblem& p, cudaStream_t stream);
// Raises shared-memory limits of the GEMM kernels on the current device.
int gemm_prepare_device();
// Forces one tile configuration (0 = automatic choice); returns the old value.
int gemm_set_variant(int v);

// Device error word of the current device (resolved once per device).
int* device_error_word();
// Streaming-multiprocessor count of the current device (cached).
int device_num_sms();

// Elementwise / normalisation launchers (elementwise.cu).
int split_tf32_launch(const float* x, int64_t rows, int cols, int64_t ldx, float* pair, int ldp,
                      cudaStream_t s);
int layernorm_launch(const float* x, int64_t ldx, const float* gamma, const float* beta,
                     float* y, int64_t ldy, float* y_pair, int64_t pair_ld, int64_t pair_plane,
                     int64_t rows, int E, float eps, cudaStream_t s);
int im2col_pair_launch(const float* img, int B, int C, int H, int W, float* pair, cudaStream_t s);
int cls_pos_launch(const float* cls, int64_t cls_stride, const float* pos, const float* patches,
                   float* out, int B, int P, int E, cudaStream_t s);
int gemm_k0_launch(const GemmProblem& p, cudaStream_t s);

// Attention (attention.cu).
int attention_launch(const float* q, const float* k, const float* v, int64_t ldq, int64_t ldk,
                     int64_t ldv, float* o, int64_t ldo, float* o_pair, int64_t pair_ld,
                     int64_t pair_plane, int B, int T, int heads, float scale, cudaStream_t s);

// Counts one kernel launch issued by the library (process-wide).
void count_launch();

// Converts a CUDA error to a status (0 stays 0).
inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? 0 : static_cast<int>(e); }

}  // namespace vitb200
