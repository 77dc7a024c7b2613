// C ABI of libvitb200.so (declared in include/vitb200.h): argument checks,
// workspace carving, per-device set-up, and the whole-model forward that chains
// the kernels on one stream.
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "engine.h"
#include "vitb200.h"

namespace vitb200 {

// Device error word: kernels that give up on a bounded wait record a code here.
static __device__ int g_error_word[4];

namespace {

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool ready = false;
  int status = 0;
  int* err = nullptr;
  int sms = 148;
};

DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

DeviceState* device_state(int* status) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *status = cuda_status(e);
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    *status = VITB200_E_UNSUPPORTED;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_dev_mu);
  DeviceState& d = g_dev[dev];
  if (!d.ready) {
    void* p = nullptr;
    int st = cuda_status(cudaGetSymbolAddress(&p, g_error_word));
    if (!st) st = cuda_status(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
    if (!st) {
      d.err = static_cast<int*>(p);
      d.ready = true;  // gemm_prepare_device() below reads the SM count
      st = gemm_prepare_device();
      if (!st) st = attention_prepare_device();
      if (!st) st = attention_f16_prepare_device();
      if (st) d.ready = false;
    }
    d.status = st;
    if (st) {
      *status = st;
      return nullptr;
    }
  }
  *status = 0;
  return &d;
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline int round4(int v) { return (v + 3) / 4 * 4; }

// Bump allocator over the caller's workspace; with base == nullptr it only
// measures.
struct Carve {
  uint8_t* base;
  size_t cap;
  size_t off = 0;
  float* take(size_t nfloats) {
    off = align_up(off, 256);
    float* p = base ? reinterpret_cast<float*>(base + off) : nullptr;
    off += nfloats * sizeof(float);
    return p;
  }
  bool fits() const { return off <= cap; }
};

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int check_ready() {
  int st = 0;
  device_state(&st);
  return st;
}

}  // namespace

static std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("VITB200_PDL");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

bool tma_store_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("VITB200_TMA_STORE");
    return !(v != nullptr && v[0] == '0');
  }();
  return on;
}

int* device_error_word() {
  int st = 0;
  DeviceState* d = device_state(&st);
  return d ? d->err : nullptr;
}

int device_num_sms() {
  int st = 0;
  DeviceState* d = device_state(&st);
  return d ? d->sms : 148;
}

}  // namespace vitb200

using namespace vitb200;

#define VITB200_GUARD_BEGIN try {
#define VITB200_GUARD_END \
  }                       \
  catch (...) {           \
    return VITB200_E_INVALID_ARG; \
  }

extern "C" {

int vitb200_version(void) { return 100; }

const char* vitb200_status_string(int status) {
  switch (status) {
    case VITB200_OK: return "ok";
    case VITB200_E_INVALID_ARG: return "invalid argument";
    case VITB200_E_UNSUPPORTED: return "unsupported shape or configuration";
    case VITB200_E_WORKSPACE: return "workspace too small";
    case VITB200_E_DEVICE_TIMEOUT: return "a kernel gave up on a bounded wait";
    case VITB200_E_NO_TMA: return "tensor-map encoding unavailable or rejected";
    case VITB200_E_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    default: break;
  }
  if (status > 0) return cudaGetErrorString(static_cast<cudaError_t>(status));
  return "unknown status";
}

int vitb200_init(void) {
  VITB200_GUARD_BEGIN
  return check_ready();
  VITB200_GUARD_END
}

int vitb200_device_error(int* code, int clear) {
  VITB200_GUARD_BEGIN
  if (!code) return VITB200_E_INVALID_ARG;
  int st = 0;
  DeviceState* d = device_state(&st);
  if (!d) return st;
  st = cuda_status(cudaDeviceSynchronize());
  if (st) return st;
  int host = 0;
  st = cuda_status(cudaMemcpy(&host, d->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (st) return st;
  *code = host;
  if (clear) st = cuda_status(cudaMemset(d->err, 0, sizeof(int)));
  return st;
  VITB200_GUARD_END
}

int vitb200_num_sms(void) { return device_num_sms(); }

uint64_t vitb200_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int vitb200_set_gemm_variant(int variant) { return gemm_set_variant(variant); }

int vitb200_set_split_k(int enable) { return gemm_set_split_k(enable); }

int vitb200_set_gemm_split(int ksplit) { return gemm_set_split(ksplit); }

int vitb200_check_wait_timeout(int kind, void* stream) {
  VITB200_GUARD_BEGIN
  if (kind != 0 && kind != 1) return VITB200_E_INVALID_ARG;
  if (int st = check_ready()) return st;
  return wait_timeout_launch(kind, as_stream(stream));
  VITB200_GUARD_END
}

int vitb200_gemm_plan(int64_t M, int K, int N, int f16, int* variant, int* ksplit) {
  VITB200_GUARD_BEGIN
  if (M <= 0 || K <= 0 || N <= 0) return VITB200_E_INVALID_ARG;
  const int pad = f16 ? 8 : 4;
  return gemm_plan(M, N, (K + pad - 1) / pad * pad, f16, variant, ksplit);
  VITB200_GUARD_END
}

int vitb200_split_tf32(const float* x, int64_t rows, int cols, int64_t ldx, float* pair, int ldp,
                       void* stream) {
  VITB200_GUARD_BEGIN
  if (rows < 0 || cols < 0 || ldp < cols || ldp % 4 != 0 || ldx < cols)
    return VITB200_E_INVALID_ARG;
  if (rows > 0 && ldp > 0 && (!x || !pair)) return VITB200_E_INVALID_ARG;
  if (int st = check_ready()) return st;
  return split_tf32_launch(x, rows, cols, ldx, pair, ldp, as_stream(stream));
  VITB200_GUARD_END
}

int vitb200_layernorm(const float* x, const float* gamma, const float* beta, float* y,
                      int64_t rows, int E, float eps, void* stream) {
  VITB200_GUARD_BEGIN
  if (rows < 0 || E <= 0 || !x || !gamma || !beta || !y) return VITB200_E_INVALID_ARG;
  if (int st = check_ready()) return st;
  return layernorm_launch(x, E, gamma, beta, y, E, nullptr, 0, 0, rows, E, eps,
                          as_stream(stream));
  VITB200_GUARD_END
}

// ---------------------------------------------------------------- GEMM

size_t vitb200_gemm_workspace_bytes(int64_t M, int K, int N) {
  if (M < 0 || K < 0 || N < 0) return 0;
  Carve c{nullptr, 0};
  const int Kp = round4(K);
  c.take(2 * static_cast<size_t>(M) * Kp);
  c.take(2 * static_cast<size_t>(N) * Kp);
  return align_up(c.off, 256);
}

static int epilogue_from_code(int code, const float* bias, const float* residual,
                              GemmEpilogue* e) {
  switch (code) {
    case VITB200_EPI_NONE: break;
    case VITB200_EPI_BIAS:
      if (!bias) return VITB200_E_INVALID_ARG;
      e->bias = bias;
      break;
    case VITB200_EPI_BIAS_GELU:
      if (!bias) return VITB200_E_INVALID_ARG;
      e->bias = bias;
      e->gelu = 1;
      break;
    case VITB200_EPI_BIAS_RESID:
      if (!bias || !residual) return VITB200_E_INVALID_ARG;
      e->bias = bias;
      e->residual = residual;
      break;
    default: return VITB200_E_INVALID_ARG;
  }
  return 0;
}

int vitb200_gemm(const float* X, const float* W, const float* bias, const float* residual,
                 float* Y, int64_t M, int K, int N, int epilogue, void* workspace,
                 size_t workspace_bytes, void* stream) {
  VITB200_GUARD_BEGIN
  if (M < 0 || K < 0 || N < 0) return VITB200_E_INVALID_ARG;
  if (epilogue < VITB200_EPI_NONE || epilogue > VITB200_EPI_BIAS_RESID) return VITB200_E_INVALID_ARG;
  if (M == 0 || N == 0) return 0;  // empty output: nothing to launch
  GemmEpilogue e;
  if (int st = epilogue_from_code(epilogue, bias, residual, &e)) return st;
  if (!Y || (K > 0 && (!X || !W))) return VITB200_E_INVALID_ARG;
  const int Kp = round4(K);
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  float* ap = c.take(2 * static_cast<size_t>(M) * Kp);
  float* wp = c.take(2 * static_cast<size_t>(N) * Kp);
  if (K > 0 && (!workspace || !c.fits())) return VITB200_E_WORKSPACE;
  if (int st = check_ready()) return st;
  cudaStream_t s = as_stream(stream);
  if (K > 0) {
    if (int st = split_tf32_launch(X, M, K, K, ap, Kp, s)) return st;
    if (int st = split_tf32_launch(W, N, K, K, wp, Kp, s)) return st;
  }
  GemmProblem p;
  p.a_pair = ap;
  p.b_pair = wp;
  p.M = M;
  p.N = N;
  p.Kp = K > 0 ? Kp : 0;
  e.ldr = N;
  e.out = Y;
  e.ldo = N;
  p.epi = e;
  return gemm_pairs_launch(p, s);
  VITB200_GUARD_END
}

int vitb200_gemm_pairs(const float* a_pair, const float* w_pair, const float* bias,
                       const float* residual, float* Y, int64_t ldy, float* y_pair, int64_t M,
                       int Kp, int N, int epilogue, void* stream) {
  VITB200_GUARD_BEGIN
  if (M < 0 || Kp < 0 || N < 0 || Kp % 4) return VITB200_E_INVALID_ARG;
  if (epilogue < VITB200_EPI_NONE || epilogue > VITB200_EPI_BIAS_RESID) return VITB200_E_INVALID_ARG;
  if (M == 0 || N == 0) return 0;
  GemmEpilogue e;
  if (int st = epilogue_from_code(epilogue, bias, residual, &e)) return st;
  if (!Y && !y_pair) return VITB200_E_INVALID_ARG;
  if (Y && ldy < N) return VITB200_E_INVALID_ARG;
  if (int st = check_ready()) return st;
  GemmProblem p;
  p.a_pair = a_pair;
  p.b_pair = w_pair;
  p.M = M;
  p.N = N;
  p.Kp = Kp;
  e.ldr = N;
  e.out = Y;
  e.ldo = ldy;
  e.out_pair = y_pair;
  e.ldp = N;
  e.pair_plane = M * static_cast<int64_t>(N);
  p.epi = e;
  return gemm_pairs_launch(p, as_stream(stream));
  VITB200_GUARD_END
}

int vitb200_split_f16(const float* x, int64_t rows, int cols, int64_t ldx, float scale,
                      uint16_t* planes, int64_t ldp, int nplanes, void* stream) {
  VITB200_GUARD_BEGIN
  if (rows < 0 || cols < 0 || ldp < cols || ldp % 8 != 0 || ldx < cols ||
      (nplanes != 2 && nplanes != 3) || !(scale > 0.f))
    return VITB200_E_INVALID_ARG;
  if (rows > 0 && ldp > 0 && (!x || !planes)) return VITB200_E_INVALID_ARG;
  if (int st = check_ready()) return st;
  return split_f16_launch(x, rows, cols, ldx, scale, planes, ldp, nplanes, as_stream(stream));
  VITB200_GUARD_END
}

int vitb200_gemm_f16(const uint16_t* a_planes, const uint16_t* w_planes, float acc_scale,
                     const float* bias, const float* residual, float* Y, int64_t ldy,
                     uint16_t* y_h16, int64_t M, int Kp, int N, int epilogue, void* stream) {
  VITB200_GUARD_BEGIN
  if (M < 0 || Kp < 0 || N < 0 || Kp % 8 || !(acc_scale > 0.f)) return VITB200_E_INVALID_ARG;
  if (epilogue < VITB200_EPI_NONE || epilogue > VITB200_EPI_BIAS_RESID) return VITB200_E_INVALID_ARG;
  if (M == 0 || N == 0) return 0;
  GemmEpilogue e;
  if (int st = epilogue_from_code(epilogue, bias, residual, &e)) return st;
  if (!Y && !y_h16) return VITB200_E_INVALID_ARG;
  if (Y && ldy < N) return VITB200_E_INVALID_ARG;
  if (int st = check_ready()) return st;
  GemmProblem p;
  p.f16 = 1;
  p.a_h16 = a_planes;
  p.b_h16 = w_planes;
  p.acc_scale = acc_scale;
  p.M = M;
  p.N = N;
  p.Kp = Kp;
  e.ldr = N;
  e.out = Y;
  e.ldo = ldy;
  e.out_h16 = y_h16;
  e.ldh = N;
  e.h16_plane = M * static_cast<int64_t>(N);
  p.epi = e;
  return gemm_pairs_launch(p, as_stream(stream));
  VITB200_GUARD_END
}

// ---------------------------------------------------------------- QKV

size_t vitb200_qkv_workspace_bytes(int64_t M, int E) {
  return vitb200_gemm_workspace_bytes(M, E, 3 * E);
}

int vitb200_qkv(const float* X, const float* W, const float* b, float* qkv_out, int64_t M, int E,
                void* workspace, size_t workspace_bytes, void* stream) {
  VITB200_GUARD_BEGIN
  if (M < 0 || E <= 0 || !b) return VITB200_E_INVALID_ARG;
  if (E % 32) return VITB200_E_UNSUPPORTED;
  if (M == 0) return 0;
  if (!X || !W || !qkv_out) return VITB200_E_INVALID_ARG;
  const int N = 3 * E, Kp = round4(E);
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  float* ap = c.take(2 * static_cast<size_t>(M) * Kp);
  float* wp = c.take(2 * static_cast<size_t>(N) * Kp);
  if (!workspace || !c.fits()) return VITB200_E_WORKSPACE;
  if (int st = check_ready()) return st;
  cudaStream_t s = as_stream(stream);
  if (int st = split_tf32_launch(X, M, E, E, ap, Kp, s)) return st;
  if (int st = split_tf32_launch(W, N, E, E, wp, Kp, s)) return st;
  GemmProblem p;
  p.a_pair = ap;
  p.b_pair = wp;
  p.M = M;
  p.N = N;
  p.Kp = Kp;
  p.epi.bias = b;
  p.epi.out = qkv_out;
  p.epi.ldo = E;
  p.epi.mode = kModeSplit3;
  p.epi.e_split = E;
  p.epi.split_plane = M * static_cast<int64_t>(E);
  return gemm_pairs_launch(p, s);
  VITB200_GUARD_END
}

// ---------------------------------------------------------------- MLP

size_t vitb200_mlp_workspace_bytes(int64_t M, int E, int E4) {
  if (M < 0 || E < 0 || E4 < 0) return 0;
  Carve c{nullptr, 0};
  const int K1 = round4(E), K2 = round4(E4);
  c.take(2 * static_cast<size_t>(M) * K1);
  c.take(2 * static_cast<size_t>(E4) * K1);
  c.take(2 * static_cast<size_t>(E) * K2);
  c.take(2 * static_cast<size_t>(M) * K2);
  return align_up(c.off, 256);
}

int vitb200_mlp(const float* X, const float* W1, const float* b1, const float* W2,
                const float* b2, float* H, float* O, int64_t M, int E, int E4, void* workspace,
                size_t workspace_bytes, void* stream) {
  VITB200_GUARD_BEGIN
  if (M < 0 || E <= 0 || E4 <= 0 || !b1 || !b2) return VITB200_E_INVALID_ARG;
  if (M == 0) return 0;
  if (!X || !W1 || !W2 || !H || !O) return VITB200_E_INVALID_ARG;
  const int K1 = round4(E), K2 = round4(E4);
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  float* xp = c.take(2 * static_cast<size_t>(M) * K1);
  float* w1p = c.take(2 * static_cast<size_t>(E4) * K1);
  float* w2p = c.take(2 * static_cast<size_t>(E) * K2);
  float* hp = c.take(2 * static_cast<size_t>(M) * K2);
  if (!workspace || !c.fits()) return VITB200_E_WORKSPACE;
  if (int st = check_ready()) return st;
  cudaStream_t s = as_stream(stream);
  if (int st = split_tf32_launch(X, M, E, E, xp, K1, s)) return st;
  if (int st = split_tf32_launch(W1, E4, E, E, w1p, K1, s)) return st;
  if (int st = split_tf32_launch(W2, E, E4, E4, w2p, K2, s)) return st;
  GemmProblem p1;
  p1.a_pair = xp;
  p1.b_pair = w1p;
  p1.M = M;
  p1.N = E4;
  p1.Kp = K1;
  p1.epi.bias = b1;
  p1.epi.gelu = 1;
  p1.epi.out = H;
  p1.epi.ldo = E4;
  if (K2 == E4) {  // the epilogue writes the hidden pair directly
    p1.epi.out_pair = hp;
    p1.epi.ldp = K2;
    p1.epi.pair_plane = M * static_cast<int64_t>(K2);
  }
  if (int st = gemm_pairs_launch(p1, s)) return st;
  if (K2 != E4) {
    if (int st = split_tf32_launch(H, M, E4, E4, hp, K2, s)) return st;
  }
  GemmProblem p2;
  p2.a_pair = hp;
  p2.b_pair = w2p;
  p2.M = M;
  p2.N = E;
  p2.Kp = K2;
  p2.epi.bias = b2;
  p2.epi.out = O;
  p2.epi.ldo = E;
  return gemm_pairs_launch(p2, s);
  VITB200_GUARD_END
}

// ---------------------------------------------------------------- attention

static size_t vt_pair_floats(int B, int T, int heads) {
  const size_t T4 = (static_cast<size_t>(T) + 3) / 4 * 4;
  return 2 * static_cast<size_t>(B) * heads * 64 * T4;
}

size_t vitb200_attention_workspace_bytes(int B, int T, int heads) {
  if (B < 0 || T < 0 || heads <= 0) return 0;
  Carve c{nullptr, 0};
  const size_t n = 2 * static_cast<size_t>(B) * T * heads * 64;
  c.take(n);
  c.take(n);
  c.take(vt_pair_floats(B, T, heads));
  return align_up(c.off, 256);
}

int vitb200_attention(const float* q, const float* k, const float* v, float* o, int B, int T,
                      int heads, int64_t ldq, int64_t ldk, int64_t ldv, int64_t ldo, float scale,
                      void* workspace, size_t workspace_bytes, void* stream) {
  VITB200_GUARD_BEGIN
  if (B < 0 || T < 0 || heads <= 0 || !q || !k || !v || !o) return VITB200_E_INVALID_ARG;
  const int64_t width = static_cast<int64_t>(heads) * 64;
  if (ldq < width || ldk < width || ldv < width || ldo < width) return VITB200_E_INVALID_ARG;
  if (B == 0 || T == 0) return 0;
  const int64_t M = static_cast<int64_t>(B) * T;
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  float* qp = c.take(2 * static_cast<size_t>(M) * width);
  float* kp = c.take(2 * static_cast<size_t>(M) * width);
  float* vtp = c.take(vt_pair_floats(B, T, heads));
  if (!workspace || !c.fits()) return VITB200_E_WORKSPACE;
  if (int st = check_ready()) return st;
  cudaStream_t s = as_stream(stream);
  const int w = static_cast<int>(width);
  if (int st = split_tf32_launch(q, M, w, ldq, qp, w, s)) return st;
  if (int st = split_tf32_launch(k, M, w, ldk, kp, w, s)) return st;
  if (int st = split_transpose_v_launch(v, ldv, B, T, heads, vtp, s)) return st;
  return attention_launch(qp, w, 0, kp, w, 0, vtp, o, ldo, nullptr, 0, 0, B, T, heads, scale, s);
  VITB200_GUARD_END
}

static size_t vt16_halves(int B, int T, int heads) {
  const size_t T8 = (static_cast<size_t>(T) + 7) / 8 * 8;
  return 2 * static_cast<size_t>(B) * heads * 64 * T8;
}

size_t vitb200_attention_f16_workspace_bytes(int B, int T, int heads) {
  if (B < 0 || T < 0 || heads <= 0) return 0;
  Carve c{nullptr, 0};
  const size_t n = static_cast<size_t>(B) * T * heads * 64;
  c.take((2 * n + 1) / 2);         // q16: 2 planes of halves
  c.take((2 * n + 1) / 2);         // k16: 2 planes
  c.take((vt16_halves(B, T, heads) + 1) / 2);
  return align_up(c.off, 256);
}

int vitb200_attention_f16(const float* q, const float* k, const float* v, float* o, int B, int T,
                          int heads, int64_t ldq, int64_t ldk, int64_t ldv, int64_t ldo,
                          float scale, float k_scale, float v_scale, void* workspace,
                          size_t workspace_bytes, void* stream) {
  VITB200_GUARD_BEGIN
  if (B < 0 || T < 0 || heads <= 0 || !q || !k || !v || !o) return VITB200_E_INVALID_ARG;
  if (!(k_scale > 0.f) || !(v_scale > 0.f)) return VITB200_E_INVALID_ARG;
  const int64_t width = static_cast<int64_t>(heads) * 64;
  if (ldq < width || ldk < width || ldv < width || ldo < width) return VITB200_E_INVALID_ARG;
  if (B == 0 || T == 0) return 0;
  const int64_t M = static_cast<int64_t>(B) * T;
  const size_t n = static_cast<size_t>(M) * width;
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  uint16_t* q16 = reinterpret_cast<uint16_t*>(c.take((2 * n + 1) / 2));
  uint16_t* k16 = reinterpret_cast<uint16_t*>(c.take((2 * n + 1) / 2));
  uint16_t* vt16 = reinterpret_cast<uint16_t*>(c.take((vt16_halves(B, T, heads) + 1) / 2));
  if (!workspace || !c.fits()) return VITB200_E_WORKSPACE;
  if (int st = check_ready()) return st;
  cudaStream_t s = as_stream(stream);
  if (int st = split_f16_launch(q, M, static_cast<int>(width), ldq, 1.f, q16, width, 2, s))
    return st;
  if (int st = split_f16_launch(k, M, static_cast<int>(width), ldk, k_scale, k16, width, 2, s))
    return st;
  if (int st = split_transpose_v_f16_launch(v, ldv, B, T, heads, v_scale, vt16, s)) return st;
  return attention_f16_launch(q16, k16, width, vt16, (T + 7) / 8 * 8, o, ldo, nullptr, 0, 0,
                              nullptr, 0, 0, B, T, heads, scale, 1.f, k_scale, v_scale, s);
  VITB200_GUARD_END
}

// ---------------------------------------------------------------- patch embed

size_t vitb200_patch_embed_workspace_bytes(int B, int C, int H, int W, int E) {
  if (B < 0 || C <= 0 || H < 16 || W < 16 || E <= 0) return 0;
  Carve c{nullptr, 0};
  const int64_t Mp = static_cast<int64_t>(B) * (H / 16) * (W / 16);
  const int K = C * 256;
  c.take(2 * static_cast<size_t>(Mp) * K);
  c.take(2 * static_cast<size_t>(E) * K);
  return align_up(c.off, 256);
}

int vitb200_patch_embed(const float* img, const float* weights, const float* bias, float* out,
                        int B, int C, int H, int W, int E, void* workspace,
                        size_t workspace_bytes, void* stream) {
  VITB200_GUARD_BEGIN
  if (B < 0 || C <= 0 || E <= 0 || H < 16 || W < 16 || H % 16 || W % 16)
    return VITB200_E_INVALID_ARG;
  if (B == 0) return 0;
  if (!img || !weights || !out) return VITB200_E_INVALID_ARG;
  const int64_t Mp = static_cast<int64_t>(B) * (H / 16) * (W / 16);
  const int K = C * 256;
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  float* ap = c.take(2 * static_cast<size_t>(Mp) * K);
  float* wp = c.take(2 * static_cast<size_t>(E) * K);
  if (!workspace || !c.fits()) return VITB200_E_WORKSPACE;
  if (int st = check_ready()) return st;
  cudaStream_t s = as_stream(stream);
  if (int st = im2col_pair_launch(img, B, C, H, W, ap, s)) return st;
  if (int st = split_tf32_launch(weights, E, K, K, wp, K, s)) return st;
  GemmProblem p;
  p.a_pair = ap;
  p.b_pair = wp;
  p.M = Mp;
  p.N = E;
  p.Kp = K;
  p.epi.bias = bias;  // optional, as in patch_embed_wrapper.cpp:46-48
  p.epi.out = out;
  p.epi.ldo = E;
  return gemm_pairs_launch(p, s);
  VITB200_GUARD_END
}

int vitb200_pos_encoding(const float* patches, const float* cls, const float* pos, float* out,
                         int B, int P, int E, void* stream) {
  VITB200_GUARD_BEGIN
  if (B < 0 || P < 0 || E <= 0 || !cls || !pos || !out) return VITB200_E_INVALID_ARG;
  if (!patches && B > 0 && P > 0) return VITB200_E_INVALID_ARG;
  if (int st = check_ready()) return st;
  return cls_pos_launch(cls, E, pos, patches, out, B, P, E, as_stream(stream));
  VITB200_GUARD_END
}

// ---------------------------------------------------------------- classifier

size_t vitb200_classifier_workspace_bytes(int B, int E, int C) {
  return vitb200_gemm_workspace_bytes(B, E, C);
}

int vitb200_classifier(const float* X, const float* W, const float* bias, float* logits, int B,
                       int T, int E, int C, void* workspace, size_t workspace_bytes,
                       void* stream) {
  VITB200_GUARD_BEGIN
  if (B < 0 || T <= 0 || E <= 0 || C < 0 || !bias) return VITB200_E_INVALID_ARG;
  if (B == 0 || C == 0) return 0;
  if (!X || !W || !logits) return VITB200_E_INVALID_ARG;
  const int Kp = round4(E);
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  float* ap = c.take(2 * static_cast<size_t>(B) * Kp);
  float* wp = c.take(2 * static_cast<size_t>(C) * Kp);
  if (!workspace || !c.fits()) return VITB200_E_WORKSPACE;
  if (int st = check_ready()) return st;
  cudaStream_t s = as_stream(stream);
  // CLS rows are every T-th row of X.
  if (int st = split_tf32_launch(X, B, E, static_cast<int64_t>(T) * E, ap, Kp, s)) return st;
  if (int st = split_tf32_launch(W, C, E, E, wp, Kp, s)) return st;
  GemmProblem p;
  p.a_pair = ap;
  p.b_pair = wp;
  p.M = B;
  p.N = C;
  p.Kp = Kp;
  p.epi.bias = bias;
  p.epi.out = logits;
  p.epi.ldo = C;
  return gemm_pairs_launch(p, s);
  VITB200_GUARD_END
}

// ---------------------------------------------------------------- model

namespace {

struct VitDims {
  int P, T, Kpatch;
  int64_t M, Mp;
};

int check_params(const vitb200_vit_params* p, int batch, VitDims* d) {
  if (!p || batch < 0) return VITB200_E_INVALID_ARG;
  if (p->embed_dim != 768 || p->num_heads * 64 != p->embed_dim || p->patch != 16)
    return VITB200_E_UNSUPPORTED;
  if (p->depth <= 0 || p->mlp_dim <= 0 || p->mlp_dim % 32 || p->in_chans <= 0 ||
      p->num_classes < 0)
    return VITB200_E_INVALID_ARG;
  if (p->img_h < 16 || p->img_w < 16 || p->img_h % 16 || p->img_w % 16)
    return VITB200_E_INVALID_ARG;
  if ((!p->patch_w_pair && !p->patch_w_f16) || !p->patch_b || !p->cls_token || !p->pos_embed ||
      !p->blocks || !p->norm_w || !p->norm_b)
    return VITB200_E_INVALID_ARG;
  if (p->patch_w_f16 && !(p->patch_acc_scale > 0.f)) return VITB200_E_INVALID_ARG;
  for (int i = 0; i < p->depth; ++i) {
    const vitb200_block_params& b = p->blocks[i];
    if (!b.norm1_w || !b.norm1_b || !b.qkv_b || !b.proj_b || !b.norm2_w || !b.norm2_b ||
        !b.fc1_b || !b.fc2_b)
      return VITB200_E_INVALID_ARG;
    if ((!b.qkv_w_pair && !b.qkv_w_f16) || (!b.proj_w_pair && !b.proj_w_f16) ||
        (!b.fc1_w_pair && !b.fc1_w_f16) || (!b.fc2_w_pair && !b.fc2_w_f16))
      return VITB200_E_INVALID_ARG;
    if ((b.qkv_w_f16 && !(b.qkv_acc_scale > 0.f)) || (b.proj_w_f16 && !(b.proj_acc_scale > 0.f)) ||
        (b.fc1_w_f16 && !(b.fc1_acc_scale > 0.f)) || (b.fc2_w_f16 && !(b.fc2_acc_scale > 0.f)))
      return VITB200_E_INVALID_ARG;
    if (b.attn_f16 && (!(b.q_scale > 0.f) || !(b.k_scale > 0.f) || !(b.v_scale > 0.f)))
      return VITB200_E_INVALID_ARG;
    if (p->ln_fold &&
        (!b.ln_qkv_w_f16 || !b.ln_qkv_c || !b.ln_qkv_d || !(b.ln_qkv_acc_scale > 0.f) ||
         !b.ln_fc1_w_f16 || !b.ln_fc1_c || !b.ln_fc1_d || !(b.ln_fc1_acc_scale > 0.f) ||
         !b.proj_w_f16 || !b.fc2_w_f16))
      return VITB200_E_INVALID_ARG;
  }
  d->P = (p->img_h / 16) * (p->img_w / 16);
  d->T = d->P + 1;
  d->Kpatch = p->in_chans * 256;
  d->M = static_cast<int64_t>(batch) * d->T;
  d->Mp = static_cast<int64_t>(batch) * d->P;
  return 0;
}

// Folded LayerNorms pay off only below this many token rows: there the 23
// LayerNorm launches they save are mostly launch latency, while at batch 256
// the residual GEMMs' extra split-and-statistics work costs more than the
// LayerNorm kernels (measured 29.46 vs 28.83 ms per forward on one B200;
// batch 1: 0.852 vs 0.877 ms). The same threshold picks CTA-pair GEMM tiles.
constexpr int64_t kLnFoldMaxRows = 1024;

bool use_ln_fold(const vitb200_vit_params* p, const VitDims& d) {
  return p->ln_fold != 0 && d.M < kLnFoldMaxRows;
}

// Workspace regions of the forward. x is the residual stream [M][768];
// pair_a holds the im2col pair, then per block the LN1 / attention / LN2
// outputs (a TF32 pair, or an FP16 split in the same space when the consuming
// GEMM runs on FP16 operands); qk the TF32 pair [2][M][1536] of q|k; vt the
// TF32 pair of V transposed per (image, head) [2][B*heads][64][T4]; hpair the
// GELU output (TF32 pair [2][M][mlp] or its FP16 split); cls_pair the final
// LN of the CLS rows.
struct VitBuffers {
  float *x, *pair_a, *qk, *vt, *hpair, *cls_pair;
  // ln_fold: the FP16 split of x [2][M][768] and its slab statistics [24][M].
  uint16_t* xs;
  float2* xstats;
};

size_t carve_vit(const vitb200_vit_params* p, const VitDims& d, int batch, Carve* c,
                 VitBuffers* b) {
  const size_t D = static_cast<size_t>(p->embed_dim);
  b->x = c->take(static_cast<size_t>(d.M) * D);
  b->pair_a = c->take(2 * std::max(static_cast<size_t>(d.M) * D,
                                   static_cast<size_t>(d.Mp) * d.Kpatch));
  // qk / vt also hold the FP16 attention's q16 + k16 (4 planes of halves) and vt16.
  b->qk = c->take(2 * static_cast<size_t>(d.M) * 2 * D);
  b->vt = c->take(std::max(vt_pair_floats(batch, d.T, p->num_heads),
                           (vt16_halves(batch, d.T, p->num_heads) + 1) / 2));
  b->hpair = c->take(2 * static_cast<size_t>(d.M) * p->mlp_dim);
  b->cls_pair = c->take(2 * static_cast<size_t>(batch) * D);
  b->xs = nullptr;
  b->xstats = nullptr;
  if (use_ln_fold(p, d)) {
    b->xs = reinterpret_cast<uint16_t*>(c->take(static_cast<size_t>(d.M) * D));
    b->xstats = reinterpret_cast<float2*>(c->take(2 * static_cast<size_t>(d.M) * (D / 32)));
  }
  return align_up(c->off, 256);
}

// patches -> FP16 split (or TF32 pair without FP16 weight planes); patch GEMM
// with bias and positional rows fused into the epilogue (rows b*T+1+p); CLS
// rows cls + pos[0]. Writes x[B*T][768].
int vit_embed(const vitb200_vit_params* p, const VitDims& d, const VitBuffers& b,
              const float* img, float* x, int batch, cudaStream_t s) {
  const int D = p->embed_dim;
  const bool f16 = p->patch_w_f16 != nullptr;
  uint16_t* a16 = reinterpret_cast<uint16_t*>(b.pair_a);
  if (int st = im2col_pair_launch(img, batch, p->in_chans, p->img_h, p->img_w,
                                  f16 ? nullptr : b.pair_a, s, p->cls_token, p->pos_embed, x, D,
                                  f16 ? a16 : nullptr))
    return st;
  GemmProblem g;
  if (f16) {
    g.f16 = 1;
    g.a_h16 = a16;
    g.b_h16 = p->patch_w_f16;
    g.acc_scale = p->patch_acc_scale;
  } else {
    g.a_pair = b.pair_a;
    g.b_pair = p->patch_w_pair;
  }
  g.M = d.Mp;
  g.N = D;
  g.Kp = d.Kpatch;
  g.epi.bias = p->patch_b;
  g.epi.out = x;
  g.epi.ldo = D;
  g.epi.mode = kModePatch;
  g.epi.P = d.P;
  g.epi.T = d.T;
  g.epi.pos = p->pos_embed;
  return gemm_pairs_launch(g, s);  // rows 1..P; im2col wrote the CLS rows
}

// One pre-LN encoder block in place on x (vit_cuda/model.py:39-60 order):
// x += proj(attn(LN1 x)); x += fc2(GELU(fc1(LN2 x))). Residual adds are fused
// into the proj / fc2 epilogues.
//
// With p->ln_fold the two LayerNorms run inside the GEMMs they feed: qkv and
// fc1 read the FP16 split of x (b.xs) with W * diag(gamma) and apply
// rstd * (acc - mean * c) + d in their epilogues from the slab statistics
// (b.xstats); proj writes that split and those statistics of the new x
// beside x, and so does fc2 when emit_next (for the next block's qkv).
// xs_ready: b.xs / b.xstats already hold x's (written by the previous fc2);
// otherwise one kernel writes them first.
int vit_block_fold(const vitb200_vit_params* p, const VitDims& d, const VitBuffers& b, int layer,
                   float* x, int batch, cudaStream_t s, bool xs_ready, bool emit_next) {
  const int D = p->embed_dim;
  const int64_t M = d.M;
  const int64_t plane = M * D;
  const int64_t hplane = M * p->mlp_dim;
  const vitb200_block_params& w = p->blocks[layer];
  uint16_t* a16 = reinterpret_cast<uint16_t*>(b.pair_a);
  uint16_t* h16 = reinterpret_cast<uint16_t*>(b.hpair);
  if (!xs_ready) {
    if (int st = xsplit_stats_launch(x, D, M, b.xs, D, plane, b.xstats, s)) return st;
  }
  // The GEMM feeding from a folded LayerNorm: A = the split of x, bias -> (c, d).
  auto set_ln = [&](GemmProblem& g, const uint16_t* wf16, float acc, const float* c,
                    const float* dd) {
    g.f16 = 1;
    g.a_h16 = b.xs;
    g.b_h16 = wf16;
    g.acc_scale = acc;
    g.epi.ln_c = c;
    g.epi.ln_d = dd;
    g.epi.ln_stats = b.xstats;
    g.epi.ln_slabs = D / 32;
    g.epi.ln_eps = p->ln_eps;
  };
  // The residual GEMM writing x (and, for the next folded LayerNorm, its split
  // and statistics).
  auto set_out = [&](GemmProblem& g, bool emit) {
    g.epi.residual = x;
    g.epi.ldr = D;
    g.epi.out = x;
    g.epi.ldo = D;
    if (emit) {
      g.epi.out_h16 = b.xs;
      g.epi.ldh = D;
      g.epi.h16_plane = plane;
      g.epi.stats_out = b.xstats;
      g.epi.h16_check = 1;
    }
  };
  const int T8 = (d.T + 7) / 8 * 8;
  uint16_t* q16 = reinterpret_cast<uint16_t*>(b.qk);
  uint16_t* k16 = q16 + 2 * plane;
  uint16_t* vt16 = reinterpret_cast<uint16_t*>(b.vt);
  {
    GemmProblem g;
    set_ln(g, w.ln_qkv_w_f16, w.ln_qkv_acc_scale, w.ln_qkv_c, w.ln_qkv_d);
    g.M = M;
    g.N = 3 * D;
    g.Kp = D;
    g.epi.e_split = D;
    g.epi.T = d.T;
    if (w.attn_f16) {
      g.epi.mode = kModeQKVAttn16;
      g.epi.q16 = q16;
      g.epi.k16 = k16;
      g.epi.vt16 = vt16;
      g.epi.vt16_plane = static_cast<int64_t>(vt16_halves(batch, d.T, p->num_heads) / 2);
      g.epi.T4 = T8;
      g.epi.q_scale = w.q_scale;
      g.epi.k_scale = w.k_scale;
      g.epi.v_scale = w.v_scale;
    } else {
      g.epi.mode = kModeQKVAttn;
      g.epi.out_pair = b.qk;
      g.epi.ldp = 2 * D;
      g.epi.pair_plane = M * 2 * D;
      g.epi.T4 = (d.T + 3) / 4 * 4;
      g.epi.vt_pair = b.vt;
      g.epi.vt_plane = static_cast<int64_t>(vt_pair_floats(batch, d.T, p->num_heads) / 2);
    }
    if (int st = gemm_pairs_launch(g, s)) return st;
  }
  if (w.attn_f16) {
    if (int st = attention_f16_launch(q16, k16, D, vt16, T8, nullptr, 0, nullptr, D, plane, a16, D,
                                      plane, batch, d.T, p->num_heads, p->attn_scale, w.q_scale,
                                      w.k_scale, w.v_scale, s))
      return st;
  } else if (int st = attention_launch(b.qk, 2 * D, 0, b.qk, 2 * D, D, b.vt, nullptr, 0, nullptr,
                                       D, plane, batch, d.T, p->num_heads, p->attn_scale, s, a16,
                                       D, plane)) {
    return st;
  }
  {
    GemmProblem g;
    g.f16 = 1;
    g.a_h16 = a16;
    g.b_h16 = w.proj_w_f16;
    g.acc_scale = w.proj_acc_scale;
    g.M = M;
    g.N = D;
    g.Kp = D;
    g.epi.bias = w.proj_b;
    set_out(g, true);
    if (int st = gemm_pairs_launch(g, s)) return st;
  }
  {
    GemmProblem g;
    set_ln(g, w.ln_fc1_w_f16, w.ln_fc1_acc_scale, w.ln_fc1_c, w.ln_fc1_d);
    g.M = M;
    g.N = p->mlp_dim;
    g.Kp = D;
    g.epi.gelu = 1;
    g.epi.out_h16 = h16;
    g.epi.ldh = p->mlp_dim;
    g.epi.h16_plane = hplane;
    if (int st = gemm_pairs_launch(g, s)) return st;
  }
  GemmProblem g;
  g.f16 = 1;
  g.a_h16 = h16;
  g.b_h16 = w.fc2_w_f16;
  g.acc_scale = w.fc2_acc_scale;
  g.M = M;
  g.N = D;
  g.Kp = p->mlp_dim;
  g.epi.bias = w.fc2_b;
  set_out(g, emit_next);
  return gemm_pairs_launch(g, s);
}

int vit_block(const vitb200_vit_params* p, const VitDims& d, const VitBuffers& b, int layer,
              float* x, int batch, cudaStream_t s) {
  const int D = p->embed_dim;
  const int64_t M = d.M;
  const int64_t plane = M * D;
  const int64_t hplane = M * p->mlp_dim;
  const vitb200_block_params& w = p->blocks[layer];
  // The same space holds either operand form of a GEMM input.
  uint16_t* a16 = reinterpret_cast<uint16_t*>(b.pair_a);
  uint16_t* h16 = reinterpret_cast<uint16_t*>(b.hpair);
  const bool f_qkv = w.qkv_w_f16 != nullptr, f_proj = w.proj_w_f16 != nullptr;
  const bool f_fc1 = w.fc1_w_f16 != nullptr, f_fc2 = w.fc2_w_f16 != nullptr;
  // GEMM input A: the TF32 pair or the FP16 split in `pair`.
  auto set_a = [](GemmProblem& g, bool f16, float* pair, const float* w_pair,
                  const uint16_t* w_f16, float acc_scale) {
    if (f16) {
      g.f16 = 1;
      g.a_h16 = reinterpret_cast<const uint16_t*>(pair);
      g.b_h16 = w_f16;
      g.acc_scale = acc_scale;
    } else {
      g.a_pair = pair;
      g.b_pair = w_pair;
    }
  };
  if (int st = layernorm_launch(x, D, w.norm1_w, w.norm1_b, nullptr, 0, f_qkv ? nullptr : b.pair_a,
                                D, plane, M, D, p->ln_eps, s, f_qkv ? a16 : nullptr, D, plane))
    return st;
  const int T8 = (d.T + 7) / 8 * 8;
  uint16_t* q16 = reinterpret_cast<uint16_t*>(b.qk);
  uint16_t* k16 = q16 + 2 * plane;
  uint16_t* vt16 = reinterpret_cast<uint16_t*>(b.vt);
  {
    GemmProblem g;
    set_a(g, f_qkv, b.pair_a, w.qkv_w_pair, w.qkv_w_f16, w.qkv_acc_scale);
    g.M = M;
    g.N = 3 * D;
    g.Kp = D;
    g.epi.bias = w.qkv_b;
    g.epi.e_split = D;
    g.epi.T = d.T;
    if (w.attn_f16) {
      g.epi.mode = kModeQKVAttn16;
      g.epi.q16 = q16;
      g.epi.k16 = k16;
      g.epi.vt16 = vt16;
      g.epi.vt16_plane = static_cast<int64_t>(vt16_halves(batch, d.T, p->num_heads) / 2);
      g.epi.T4 = T8;
      g.epi.q_scale = w.q_scale;
      g.epi.k_scale = w.k_scale;
      g.epi.v_scale = w.v_scale;
    } else {
      g.epi.mode = kModeQKVAttn;
      g.epi.out_pair = b.qk;
      g.epi.ldp = 2 * D;
      g.epi.pair_plane = M * 2 * D;
      g.epi.T4 = (d.T + 3) / 4 * 4;
      g.epi.vt_pair = b.vt;
      g.epi.vt_plane = static_cast<int64_t>(vt_pair_floats(batch, d.T, p->num_heads) / 2);
    }
    if (int st = gemm_pairs_launch(g, s)) return st;
  }
  if (w.attn_f16) {
    if (int st = attention_f16_launch(q16, k16, D, vt16, T8, nullptr, 0,
                                      f_proj ? nullptr : b.pair_a, D, plane,
                                      f_proj ? a16 : nullptr, D, plane, batch, d.T,
                                      p->num_heads, p->attn_scale, w.q_scale, w.k_scale,
                                      w.v_scale, s))
      return st;
  } else if (int st = attention_launch(b.qk, 2 * D, 0, b.qk, 2 * D, D, b.vt, nullptr, 0,
                                       f_proj ? nullptr : b.pair_a, D, plane, batch, d.T,
                                       p->num_heads, p->attn_scale, s, f_proj ? a16 : nullptr, D,
                                       plane)) {
    return st;
  }
  {
    GemmProblem g;
    set_a(g, f_proj, b.pair_a, w.proj_w_pair, w.proj_w_f16, w.proj_acc_scale);
    g.M = M;
    g.N = D;
    g.Kp = D;
    g.epi.bias = w.proj_b;
    g.epi.residual = x;
    g.epi.ldr = D;
    g.epi.out = x;
    g.epi.ldo = D;
    if (int st = gemm_pairs_launch(g, s)) return st;
  }
  if (int st = layernorm_launch(x, D, w.norm2_w, w.norm2_b, nullptr, 0, f_fc1 ? nullptr : b.pair_a,
                                D, plane, M, D, p->ln_eps, s, f_fc1 ? a16 : nullptr, D, plane))
    return st;
  {
    GemmProblem g;
    set_a(g, f_fc1, b.pair_a, w.fc1_w_pair, w.fc1_w_f16, w.fc1_acc_scale);
    g.M = M;
    g.N = p->mlp_dim;
    g.Kp = D;
    g.epi.bias = w.fc1_b;
    g.epi.gelu = 1;
    if (f_fc2) {
      g.epi.out_h16 = h16;
      g.epi.ldh = p->mlp_dim;
      g.epi.h16_plane = hplane;
    } else {
      g.epi.out_pair = b.hpair;
      g.epi.ldp = p->mlp_dim;
      g.epi.pair_plane = hplane;
    }
    if (int st = gemm_pairs_launch(g, s)) return st;
  }
  GemmProblem g;
  set_a(g, f_fc2, b.hpair, w.fc2_w_pair, w.fc2_w_f16, w.fc2_acc_scale);
  g.M = M;
  g.N = D;
  g.Kp = p->mlp_dim;
  g.epi.bias = w.fc2_b;
  g.epi.residual = x;
  g.epi.ldr = D;
  g.epi.out = x;
  g.epi.ldo = D;
  return gemm_pairs_launch(g, s);
}

// The encoder blocks in order; with folded LayerNorms each fc2 hands the next
// block's qkv the split and statistics of x.
int vit_blocks(const vitb200_vit_params* p, const VitDims& d, const VitBuffers& b, float* x,
               int batch, cudaStream_t s) {
  const bool fold = use_ln_fold(p, d);
  for (int i = 0; i < p->depth; ++i) {
    const int st = fold ? vit_block_fold(p, d, b, i, x, batch, s, i > 0, i + 1 < p->depth)
                        : vit_block(p, d, b, i, x, batch, s);
    if (st) return st;
  }
  return 0;
}

// Final LayerNorm on the CLS rows only (the head reads token 0 alone) and the
// head: one fused kernel (CUDA-core FP32 dot products, batch invariant; at
// batch 1 a head GEMM launch is all latency), with LayerNorm + head GEMM for
// what it does not cover (E != 768, over 524,280 images). features / logits
// may each be null.
constexpr int kFusedHeadMaxBatch = 65535 * 8;

int vit_head(const vitb200_vit_params* p, const VitDims& d, const VitBuffers& b, const float* x,
             float* logits, float* features, int batch, cudaStream_t s) {
  const int D = p->embed_dim;
  const int64_t cls_stride = static_cast<int64_t>(d.T) * D;
  const bool want_logits = logits != nullptr && p->num_classes > 0;
  if (!features && !want_logits) return 0;
  if (want_logits && batch <= kFusedHeadMaxBatch && D == 768 && cls_stride % 4 == 0)
    return cls_head_launch(x, cls_stride, p->norm_w, p->norm_b, p->ln_eps, p->head_w_pair,
                           p->head_b, p->num_classes, D, batch, logits, features, s);
  if (int st = layernorm_launch(x, cls_stride, p->norm_w, p->norm_b, features, D,
                                want_logits ? b.cls_pair : nullptr, D,
                                static_cast<int64_t>(batch) * D, batch, D, p->ln_eps, s))
    return st;
  if (!want_logits) return 0;
  GemmProblem g;
  g.a_pair = b.cls_pair;
  g.b_pair = p->head_w_pair;
  g.M = batch;
  g.N = p->num_classes;
  g.Kp = D;
  g.epi.bias = p->head_b;
  g.epi.out = logits;
  g.epi.ldo = p->num_classes;
  return gemm_pairs_launch(g, s);
}

// Shared prologue of the model entry points: checks, device set-up, carving.
int vit_prepare(const vitb200_vit_params* p, int batch, void* workspace, size_t workspace_bytes,
                VitDims* d, VitBuffers* b) {
  if (int st = check_params(p, batch, d)) return st;
  Carve c{static_cast<uint8_t*>(workspace), workspace_bytes};
  carve_vit(p, *d, batch, &c, b);
  if (batch > 0 && (!workspace || !c.fits())) return VITB200_E_WORKSPACE;
  return check_ready();
}

}  // namespace

size_t vitb200_vit_workspace_bytes(const vitb200_vit_params* p, int batch) {
  VitDims d;
  if (check_params(p, batch, &d)) return 0;
  Carve c{nullptr, 0};
  VitBuffers b;
  return carve_vit(p, d, batch, &c, &b);
}

int vitb200_vit_forward(const vitb200_vit_params* p, const float* img, float* logits, int batch,
                        void* workspace, size_t workspace_bytes, void* stream) {
  VITB200_GUARD_BEGIN
  if (!logits || !img) return VITB200_E_INVALID_ARG;
  if (p && (!p->head_w_pair || !p->head_b)) return VITB200_E_INVALID_ARG;
  VitDims d;
  VitBuffers b;
  if (int st = vit_prepare(p, batch, workspace, workspace_bytes, &d, &b)) return st;
  if (batch == 0) return 0;
  cudaStream_t s = as_stream(stream);
  if (int st = vit_embed(p, d, b, img, b.x, batch, s)) return st;
  if (int st = vit_blocks(p, d, b, b.x, batch, s)) return st;
  return vit_head(p, d, b, b.x, logits, nullptr, batch, s);
  VITB200_GUARD_END
}

int vitb200_vit_forward_features(const vitb200_vit_params* p, const float* img, float* features,
                                 int batch, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  VITB200_GUARD_BEGIN
  if (!features || !img) return VITB200_E_INVALID_ARG;
  VitDims d;
  VitBuffers b;
  if (int st = vit_prepare(p, batch, workspace, workspace_bytes, &d, &b)) return st;
  if (batch == 0) return 0;
  cudaStream_t s = as_stream(stream);
  if (int st = vit_embed(p, d, b, img, b.x, batch, s)) return st;
  if (int st = vit_blocks(p, d, b, b.x, batch, s)) return st;
  return vit_head(p, d, b, b.x, nullptr, features, batch, s);
  VITB200_GUARD_END
}

int vitb200_vit_embed(const vitb200_vit_params* p, const float* img, float* x, int batch,
                      void* workspace, size_t workspace_bytes, void* stream) {
  VITB200_GUARD_BEGIN
  if (!img || !x) return VITB200_E_INVALID_ARG;
  VitDims d;
  VitBuffers b;
  if (int st = vit_prepare(p, batch, workspace, workspace_bytes, &d, &b)) return st;
  if (batch == 0) return 0;
  return vit_embed(p, d, b, img, x, batch, as_stream(stream));
  VITB200_GUARD_END
}

int vitb200_vit_block(const vitb200_vit_params* p, int layer, float* x, int batch,
                      void* workspace, size_t workspace_bytes, void* stream) {
  VITB200_GUARD_BEGIN
  if (!x || !p || layer < 0 || layer >= p->depth) return VITB200_E_INVALID_ARG;
  VitDims d;
  VitBuffers b;
  if (int st = vit_prepare(p, batch, workspace, workspace_bytes, &d, &b)) return st;
  if (batch == 0) return 0;
  if (use_ln_fold(p, d))
    return vit_block_fold(p, d, b, layer, x, batch, as_stream(stream), false, false);
  return vit_block(p, d, b, layer, x, batch, as_stream(stream));
  VITB200_GUARD_END
}

int vitb200_vit_head(const vitb200_vit_params* p, const float* x, float* logits,
                     float* features, int batch, void* workspace, size_t workspace_bytes,
                     void* stream) {
  VITB200_GUARD_BEGIN
  if (!x || (!logits && !features)) return VITB200_E_INVALID_ARG;
  if (p && logits && (!p->head_w_pair || !p->head_b)) return VITB200_E_INVALID_ARG;
  VitDims d;
  VitBuffers b;
  if (int st = vit_prepare(p, batch, workspace, workspace_bytes, &d, &b)) return st;
  if (batch == 0) return 0;
  return vit_head(p, d, b, x, logits, features, batch, as_stream(stream));
  VITB200_GUARD_END
}

}  // extern "C"
