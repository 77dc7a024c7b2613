// Internal host-side interfaces between the translation units of libvitb200.so.
// Not part of the C ABI (that is include/vitb200.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

namespace vitb200 {

// Row/column mapping of a GEMM epilogue.
enum EpiMode : int {
  kModePlain = 0,  // out row = m
  kModePatch = 1,  // out row = (m / P) * T + 1 + m % P, adds pos[(1 + m % P)][n]
  kModeSplit3 = 2, // column n goes to plane n / e_split, column n % e_split
  kModeQKVAttn = 3, // q|k columns -> TF32 pair rows [2][M][2E]; v columns -> the
                    // per-head transposed pair vt[2][B*heads][64][T4] (attention's V^T)
  kModeQKVAttn16 = 4, // FP16 splits for the FP16 attention: q*q_scale -> q16[2][M][E];
                      // k*k_scale -> k16[2][M][E]; v*v_scale transposed per (image,
                      // head) -> vt16[2][B*heads][64][T4] (T4 = T rounded up to 8 here)
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
  int e_split = 0;                  // kModeSplit3 / kModeQKVAttn: E
  int64_t split_plane = 0;          // kModeSplit3: elements between planes
  float* vt_pair = nullptr;         // kModeQKVAttn: [2][B*heads][64][T4]
  int64_t vt_plane = 0;             // kModeQKVAttn: elements between vt planes
  int T4 = 0;                       // kModeQKVAttn: T rounded up to 4
  uint16_t* out_h16 = nullptr;      // FP16 split of the result, planes hi | lo, or null
  int64_t ldh = 0;                  // FP16-split row stride (% 8 == 0 for 16-byte rows)
  int64_t h16_plane = 0;            // elements between the hi and lo planes
  uint16_t* q16 = nullptr;          // kModeQKVAttn16 outputs (see EpiMode)
  uint16_t* k16 = nullptr;
  uint16_t* vt16 = nullptr;
  int64_t vt16_plane = 0;           // elements between vt16 planes
  float q_scale = 1.f, k_scale = 1.f, v_scale = 1.f;  // powers of two
  // LayerNorm folded into this GEMM: A is the FP16 split of the rows x before
  // normalisation and B the planes of W * diag(gamma); the result is
  // rstd * (acc - mean * ln_c[n]) + ln_d[n] (in place of the bias), the row's
  // mean and 1 / sqrt(var + ln_eps) combined from ln_stats[s][m] = (sum, M2)
  // over the ln_slabs 32-column slabs of the row.
  const float* ln_c = nullptr;
  const float* ln_d = nullptr;
  const float2* ln_stats = nullptr;
  int ln_slabs = 0;
  float ln_eps = 0.f;
  // Statistics of the result for a LayerNorm folded into the next GEMM:
  // stats_out[n / 32][m] = (sum, M2 about the slab's mean) of each row's
  // 32-column slab; with stats_out and h16_check, a result (its FP16 split in
  // out_h16) of magnitude 32768 or more, or NaN, sets the device error.
  float2* stats_out = nullptr;
  int h16_check = 0;
};

struct GemmProblem {
  const float* a_pair = nullptr;  // TF32: [2][M][Kp]
  const float* b_pair = nullptr;  // TF32: [2][N][Kp]
  int f16 = 0;                    // 1: FP16-split operands below instead
  const uint16_t* a_h16 = nullptr;  // F16: [2][M][Kp] planes hi, lo (lo scaled by 2^11)
  const uint16_t* b_h16 = nullptr;  // F16: [3][N][Kp] planes hi, lo * 2^11, hi * 2^11
  float acc_scale = 1.f;          // F16: 2^-11 / (the scale B was split with)
  int64_t M = 0;
  int N = 0;
  int Kp = 0;                     // % 4 == 0 (TF32), % 8 == 0 (F16)
  GemmEpilogue epi;
};

// Encodes a tiled fp32 TMA tensor map of `rank` dims (innermost first; strides
// in bytes for dims 1..rank-1) with the 128-byte swizzle (64-byte if
// swizzle128 == 0). Returns a vitb200 status code.
int encode_tmap(CUtensorMap* map, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides, const uint32_t* box, int swizzle128);

// Same with FP16 elements when f16 != 0.
int encode_tmap_typed(CUtensorMap* map, int rank, const void* base, const uint64_t* dims,
                      const uint64_t* strides, const uint32_t* box, int swizzle128, int f16);

// Encodes a TMA tensor map over a TF32 pair [2][rows][Kp] with box
// [2][box_rows][BK] and the swizzle of a BK*4-byte row.
int make_pair_map(CUtensorMap* map, const float* pair, int64_t rows, int Kp, int box_rows,
                  int BK);
// Tensor map over [planes][rows][Kp] (fp32, or fp16 when f16 != 0), box = all
// planes x box_rows x BK, swizzle of one BK-element row.
int make_planes_map(CUtensorMap* map, const void* base, int64_t rows, int Kp, int planes,
                    int box_rows, int BK, int f16);

// Launches the tcgen05 GEMM (TF32x3 on TF32 pairs, or the three-product FP16
// split); returns a vitb200 status code.
int gemm_pairs_launch(const GemmProblem& p, cudaStream_t stream);
// Raises shared-memory limits of the GEMM kernels on the current device.
int gemm_prepare_device();
// Forces one tile configuration (0 = automatic choice); returns the old value.
int gemm_set_variant(int v);
// Launches a kernel whose bounded wait never completes (kind 0: a pipeline
// wait, error code 1; 1: a split-K owner's cluster-scope wait, code 7).
int wait_timeout_launch(int kind, cudaStream_t s);
// Switches split-K of later small single-CTA launches on / off; returns the
// old setting.
int gemm_set_split_k(int enable);
// Forces the K split of later small single-CTA launches to d where it fits
// (0 = automatic choice); returns the old value.
int gemm_set_split(int d);
// Tile configuration (variant) and K split a launch of this shape would use
// on the current device.
int gemm_plan(int64_t M, int N, int Kp, int f16, int* variant, int* ksplit);

// Device error word of the current device (resolved once per device).
int* device_error_word();
// Streaming-multiprocessor count of the current device (cached).
int device_num_sms();

// Elementwise / normalisation launchers (elementwise.cu).
int split_tf32_launch(const float* x, int64_t rows, int cols, int64_t ldx, float* pair, int ldp,
                      cudaStream_t s);
// x[rows][cols] * scale -> FP16 split planes out[nplanes][rows][ldo] (hi, lo*2^11,
// and with nplanes == 3 hi*2^11); columns cols..ldo-1 are zero filled. Values
// whose scaled magnitude reaches the split's limit raise the device error.
int split_f16_launch(const float* x, int64_t rows, int cols, int64_t ldx, float scale,
                     uint16_t* out, int64_t ldo, int nplanes, cudaStream_t s);
int layernorm_launch(const float* x, int64_t ldx, const float* gamma, const float* beta,
                     float* y, int64_t ldy, float* y_pair, int64_t pair_ld, int64_t pair_plane,
                     int64_t rows, int E, float eps, cudaStream_t s, uint16_t* y_h16 = nullptr,
                     int64_t h16_ld = 0, int64_t h16_plane = 0);
// Final LayerNorm of each image's CLS row (rows x + b * cls_stride, E = 768)
// fused with the head (TF32 pair [2][C][768] + bias) for small batches:
// logits [batch][C] and optionally the normalised features [batch][768].
int cls_head_launch(const float* x, int64_t cls_stride, const float* gamma, const float* beta,
                    float eps, const float* w_pair, const float* bias, int C, int E, int batch,
                    float* logits, float* features, cudaStream_t s);
// im2col into the TF32 pair (or, with h16, the FP16 split [2][B*P][C*256]);
// with x, also the CLS rows x[b][0] = cls + pos[0] of the [B][P+1][E] token
// matrix.
int im2col_pair_launch(const float* img, int B, int C, int H, int W, float* pair, cudaStream_t s,
                       const float* cls = nullptr, const float* pos = nullptr,
                       float* x = nullptr, int E = 0, uint16_t* h16 = nullptr);
int cls_pos_launch(const float* cls, int64_t cls_stride, const float* pos, const float* patches,
                   float* out, int B, int P, int E, cudaStream_t s);
int gemm_k0_launch(const GemmProblem& p, cudaStream_t s);

// Raises the attention kernel's shared-memory limit on the current device.
int attention_prepare_device();

// Attention (attention.cu) on TF32 pairs, writing fp32 O, its TF32 pair and/or
// its FP16 split. q_pair / k_pair are [2][B*T][ld]
// buffers (they may be the same buffer), head h of q at columns q_col + h*64.., of
// k at k_col + h*64..; vt_pair is V transposed per (image, head),
// [2][B*heads][64][T4] with T4 = T rounded up to 4.
int attention_launch(const float* q_pair, int64_t q_ld, int q_col, const float* k_pair,
                     int64_t k_ld, int k_col, const float* vt_pair, float* o, int64_t ldo,
                     float* o_pair, int64_t pair_ld, int64_t pair_plane, int B, int T, int heads,
                     float scale, cudaStream_t s, uint16_t* o_h16 = nullptr, int64_t h16_ld = 0,
                     int64_t h16_plane = 0);
// FP16-split attention (attention_f16.cu): q16, k16 [2][B*T][ld] (head h at
// columns h*64..), vt16 [2][B*heads][64][T8] as the QKV epilogue's
// kModeQKVAttn16 writes them (q, k, v multiplied by q_scale, k_scale, v_scale,
// powers of two). Writes fp32 O, its TF32 pair and/or its FP16 split.
int attention_f16_prepare_device();
int attention_f16_launch(const uint16_t* q16, const uint16_t* k16, int64_t ld, const uint16_t* vt16,
                         int T8, float* o, int64_t ldo, float* o_pair, int64_t pair_ld,
                         int64_t pair_plane, uint16_t* o_h16, int64_t h16_ld, int64_t h16_plane,
                         int B, int T, int heads, float scale, float q_scale, float k_scale,
                         float v_scale, cudaStream_t s);
// v[B*T][ldv] * scale -> vt16 [2][B*heads][64][T8] (hi, lo*2^11).
int split_transpose_v_f16_launch(const float* v, int64_t ldv, int B, int T, int heads, float scale,
                                 uint16_t* vt16, cudaStream_t s);
// V[B*T][ldv] (head h at columns h*64..) -> vt pair [2][B*heads][64][T4].
int split_transpose_v_launch(const float* v, int64_t ldv, int B, int T, int heads, float* vt_pair,
                             cudaStream_t s);

// Counts one kernel launch issued by the library (process-wide).
void count_launch();

// Converts a CUDA error to a status (0 stays 0).
inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? 0 : static_cast<int>(e); }

// Whether kernels are launched with programmatic stream serialization (see
// griddep_wait in common.cuh); on unless the environment sets VITB200_PDL=0.
bool pdl_enabled();

// FP16 split of x[rows][768] (planes [2][rows][hld]) and its per-row
// statistics over 32-column slabs, stats[24][rows] = (sum, M2): the input of
// a LayerNorm folded into the next GEMM. Returns a vitb200 status code.
int xsplit_stats_launch(const float* x, int64_t ldx, int64_t rows, uint16_t* h16, int64_t hld,
                        int64_t hplane, float2* stats, cudaStream_t s);

// Whether epilogues write their results through TMA tensor stores where they
// can; on unless the environment sets VITB200_TMA_STORE=0.
bool tma_store_enabled();

// Launches `kernel` on `s` with the library's launch attributes: programmatic
// stream serialization (when enabled) and, for cluster_x > 1, a cluster of
// cluster_x CTAs. Counts the launch; returns a vitb200 status code.
template <typename... KArgs, typename... Args>
int launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                  unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const int st = cuda_status(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
  count_launch();
  return st;
}

}  // namespace vitb200
