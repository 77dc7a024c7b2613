// vitb200_gemm_noalloc: the TF32x3 GEMM of vitb200_gemm for callers that
// cannot allocate device memory.
//
// vitb200_gemm needs scratch space for the TF32 hi/lo pairs of X and W and
// takes it from a caller-provided workspace. Some callers have no way to
// provide one: a plain C program or a ctypes script that owns no device
// allocator; a host whose device memory belongs to another framework's pool
// that must not be bypassed; a request path on which cudaMalloc's implicit
// device-wide synchronisation is not acceptable. This entry point keeps the
// scratch in a fixed array compiled into the library instead, so a call
// allocates nothing: no cudaMalloc, no cudaFree, no allocating library routine.
//
// Limits and sharing:
//  * the array holds kScratchFloats floats (16 MiB). Every GPU on which the
//    library is loaded keeps it resident until the process exits;
//  * a problem fits when 2*M*Kp (rounded up to 64 floats) + 2*N*Kp <= 4,194,304
//    with Kp = K rounded up to a multiple of 4, e.g. M = N = K = 1024; larger
//    problems are rejected with VITB200_E_WORKSPACE before anything is launched;
//  * every call on a device uses the same array. Calls whose GPU work may
//    overlap (different streams without ordering between them, or several host
//    threads) race on it and corrupt each other's results; calls on one stream
//    are ordered and safe. The array keeps the previous call's contents; nothing
//    needs to start at zero because the split kernel rewrites every element the
//    GEMM reads, including the zero padding of K up to Kp.
//  * the first call on a device resolves the array's device address (set-up,
//    see scratch_on_current_device); make that first call before any stream
//    capture begins. The address is cached per device ordinal for the life of
//    the process: after a cudaDeviceReset the cached address is stale, so a
//    process that resets a device must not call this entry point on it again.
#include <mutex>

#include "engine.h"
#include "vitb200.h"

namespace vitb200 {
namespace {

constexpr size_t kScratchFloats = size_t(1) << 22;  // 16 MiB of fp32
constexpr int kMaxDevices = 64;

// In host code this name is only a stand-in for the device array; its device
// address comes from cudaGetSymbolAddress below and is what the kernels get.
static __device__ __align__(256) float g_noalloc_scratch[kScratchFloats];

float* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Set-up, once per device with that device current: the device address of the
// scratch array.
int scratch_on_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return VITB200_E_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return 0;
}

inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace
}  // namespace vitb200

using namespace vitb200;

extern "C" int vitb200_gemm_noalloc(const float* X, const float* W, const float* bias,
                                    const float* residual, float* Y, int64_t M, int K, int N,
                                    int epilogue, void* stream) {
  try {
    if (M < 0 || K < 0 || N < 0) return VITB200_E_INVALID_ARG;
    if (epilogue < VITB200_EPI_NONE || epilogue > VITB200_EPI_BIAS_RESID)
      return VITB200_E_INVALID_ARG;
    if (M == 0 || N == 0) return 0;
    if ((epilogue != VITB200_EPI_NONE && !bias) ||
        (epilogue == VITB200_EPI_BIAS_RESID && !residual))
      return VITB200_E_INVALID_ARG;
    if (!Y || (K > 0 && (!X || !W))) return VITB200_E_INVALID_ARG;
    // Size check before any multiplication that could wrap: each of X's and
    // W's pairs must fit in the array on its own before the sum is formed.
    const size_t Kp = (static_cast<size_t>(K) + 3) / 4 * 4;
    const size_t half = kScratchFloats / 2;
    if (Kp > 0 && (static_cast<size_t>(M) > half / Kp || static_cast<size_t>(N) > half / Kp))
      return VITB200_E_WORKSPACE;
    const size_t a_floats = round_up(2 * static_cast<size_t>(M) * Kp, 64);
    const size_t need = a_floats + 2 * static_cast<size_t>(N) * Kp;
    if (need > kScratchFloats) return VITB200_E_WORKSPACE;
    if (int st = vitb200_init()) return st;
    float* scratch = nullptr;
    if (int st = scratch_on_current_device(&scratch)) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* ap = scratch;
    float* wp = scratch + a_floats;
    if (K > 0) {
      if (int st = split_tf32_launch(X, M, K, K, ap, static_cast<int>(Kp), s)) return st;
      if (int st = split_tf32_launch(W, N, K, K, wp, static_cast<int>(Kp), s)) return st;
    }
    GemmProblem p;
    p.a_pair = ap;
    p.b_pair = wp;
    p.M = M;
    p.N = N;
    p.Kp = K > 0 ? static_cast<int>(Kp) : 0;
    if (epilogue != VITB200_EPI_NONE) p.epi.bias = bias;
    p.epi.gelu = epilogue == VITB200_EPI_BIAS_GELU;
    if (epilogue == VITB200_EPI_BIAS_RESID) {
      p.epi.residual = residual;
      p.epi.ldr = N;
    }
    p.epi.out = Y;
    p.epi.ldo = N;
    return gemm_pairs_launch(p, s);
  } catch (...) {
    return VITB200_E_INVALID_ARG;
  }
}
