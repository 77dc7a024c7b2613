// HBM-bound kernels of the ViT path: TF32 split, LayerNorm (fp32 and/or TF32
// pair output), patch im2col into a TF32 pair, CLS + positional rows, and the
// epilogue-only GEMM for K = 0.
#include <algorithm>

#include "common.cuh"
#include "engine.h"
#include "vitb200.h"

namespace vitb200 {

namespace {

inline int grid_for(int64_t work, int threads) {
  const int64_t per_sm = 2048 / threads;
  const int64_t cap = static_cast<int64_t>(device_num_sms()) * per_sm * 4;
  const int64_t g = (work + threads - 1) / threads;
  return static_cast<int>(std::max<int64_t>(1, std::min(g, cap)));
}

}  // namespace

// ------------------------------------------------------------------ split
// pair[2][rows][ldp] <- TF32 hi/lo of x[rows][cols] (row stride ldx), zero pad.
__global__ void split_tf32_kernel(const float* __restrict__ x, int64_t rows, int cols,
                                  int64_t ldx, float* __restrict__ pair, int ldp, int vec_in) {
  griddep_wait();
  griddep_launch_dependents();
  const int q_per_row = ldp / 4;
  const int64_t total = rows * q_per_row;
  const int64_t plane = rows * ldp;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / q_per_row;
    const int c0 = static_cast<int>(i - r * q_per_row) * 4;
    const float* src = x + r * ldx + c0;
    float v[4];
    if (vec_in && c0 + 4 <= cols) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(src));
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = (c0 + j < cols) ? src[j] : 0.f;
    }
    float hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) tf32_split(v[j], hi[j], lo[j]);
    float* dst = pair + r * ldp + c0;
    *reinterpret_cast<float4*>(dst) = make_float4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<float4*>(dst + plane) = make_float4(lo[0], lo[1], lo[2], lo[3]);
  }
}

int split_tf32_launch(const float* x, int64_t rows, int cols, int64_t ldx, float* pair, int ldp,
                      cudaStream_t s) {
  if (rows < 0 || cols < 0 || ldp < cols || ldp % 4 != 0 || ldx < cols)
    return VITB200_E_INVALID_ARG;
  if (rows == 0 || ldp == 0) return 0;
  if (!x || !pair) return VITB200_E_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(pair) % 16) return VITB200_E_ALIGNMENT;
  const int vec_in = (reinterpret_cast<uintptr_t>(x) % 16 == 0) && (ldx % 4 == 0);
  const int64_t work = rows * (ldp / 4);
  if (int st_ = launch_kernel(split_tf32_kernel, dim3(grid_for(work, 256)), dim3(256), 0, s, 1, x,
      rows, cols, ldx, pair, ldp, vec_in))
    return st_;
  return cuda_status(cudaGetLastError());
}

// x[rows][cols] * scale -> FP16 split planes out[nplanes][rows][ldo]: hi,
// lo * 2^11 and (nplanes == 3) hi * 2^11; zero past cols. Eight columns per
// thread (one 16-byte store per plane).
__global__ void split_f16_kernel(const float* __restrict__ x, int64_t rows, int cols, int64_t ldx,
                                 float scale, uint16_t* __restrict__ out, int64_t ldo,
                                 int nplanes, int* err) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t o_per_row = ldo / 8;
  const int64_t total = rows * o_per_row;
  const int64_t plane = rows * ldo;
  // hi * 2^11 (the third plane) is finite only for |hi| < 32.
  const float limit = nplanes == 3 ? 16.f : kH16Limit;
  bool bad = false;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / o_per_row;
    const int c0 = static_cast<int>(i - r * o_per_row) * 8;
    const float* src = x + r * ldx + c0;
    uint32_t hw[4], lw[4], sw[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      __half h[2], l[2], s[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int c = c0 + 2 * t + u;
        const float v = (c < cols) ? __fmul_rn(src[2 * t + u], scale) : 0.f;
        bad |= !(fabsf(v) < limit);
        h16_split(v, h[u], l[u]);
        s[u] = __float2half_rn(__fmul_rn(__half2float(h[u]), kH16LoScale));
      }
      hw[t] = pack_h2(h[0], h[1]);
      lw[t] = pack_h2(l[0], l[1]);
      sw[t] = pack_h2(s[0], s[1]);
    }
    uint16_t* dst = out + r * ldo + c0;
    *reinterpret_cast<uint4*>(dst) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(dst + plane) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    if (nplanes == 3)
      *reinterpret_cast<uint4*>(dst + 2 * plane) = make_uint4(sw[0], sw[1], sw[2], sw[3]);
  }
  if (bad) report_error(err, kErrF16Range);
}

int split_f16_launch(const float* x, int64_t rows, int cols, int64_t ldx, float scale,
                     uint16_t* out, int64_t ldo, int nplanes, cudaStream_t s) {
  if (rows < 0 || cols < 0 || ldo < cols || ldo % 8 != 0 || ldx < cols ||
      (nplanes != 2 && nplanes != 3) || !(scale > 0.f))
    return VITB200_E_INVALID_ARG;
  if (rows == 0 || ldo == 0) return 0;
  if (!x || !out) return VITB200_E_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(out) % 16) return VITB200_E_ALIGNMENT;
  int* err = device_error_word();
  if (err == nullptr) return VITB200_E_INVALID_ARG;
  const int64_t work = rows * (ldo / 8);
  if (int st_ = launch_kernel(split_f16_kernel, dim3(grid_for(work, 256)), dim3(256), 0, s, 1, x,
      rows, cols, ldx, scale, out, ldo, nplanes, err))
    return st_;
  return cuda_status(cudaGetLastError());
}

// -------------------------------------------------------------- layernorm
// One warp per row. Mean, then the biased variance of (x - mean), as
// csrc/kernels/layernorm.cu:44-64 does, with an IEEE 1/sqrt instead of the
// approximate rsqrtf so results track torch's layer_norm.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// E = 768: the row lives in registers (6 float4 per lane), read once.
// LayerNorm of one 768-wide row by one warp: lane holds float4 columns
// lane + 32 i (i < 6) of x in v and gets the normalised values in o.
__device__ __forceinline__ void layernorm768_row(const float4 (&v)[6], const float4 (&g)[6],
                                                 const float4 (&b)[6], float eps,
                                                 float4 (&o)[6]) {
  constexpr int E = 768;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 6; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  const float mean = warp_sum(s) / static_cast<float>(E);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    const float a0 = v[i].x - mean, a1 = v[i].y - mean, a2 = v[i].z - mean, a3 = v[i].w - mean;
    q += (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
  }
  const float var = warp_sum(q) / static_cast<float>(E);
  const float rstd = 1.0f / sqrtf(var + eps);
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    o[i].x = (v[i].x - mean) * rstd * g[i].x + b[i].x;
    o[i].y = (v[i].y - mean) * rstd * g[i].y + b[i].y;
    o[i].z = (v[i].z - mean) * rstd * g[i].z + b[i].z;
    o[i].w = (v[i].w - mean) * rstd * g[i].w + b[i].w;
  }
}

__global__ void __launch_bounds__(256) layernorm768_kernel(
    const float* __restrict__ x, int64_t ldx, const float* __restrict__ gamma,
    const float* __restrict__ beta, float* __restrict__ y, int64_t ldy, float* __restrict__ yp,
    int64_t pld, int64_t pplane, uint16_t* __restrict__ yh, int64_t hld, int64_t hplane,
    int64_t rows, float eps) {
  griddep_wait();
  griddep_launch_dependents();
  constexpr int E = 768;
  constexpr int V = E / 128;  // float4 per lane
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  float4 g[V], b[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    g[i] = __ldg(reinterpret_cast<const float4*>(gamma) + lane + 32 * i);
    b[i] = __ldg(reinterpret_cast<const float4*>(beta) + lane + 32 * i);
  }
  for (int64_t r = warp_global; r < rows; r += nwarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + r * ldx);
    float4 v[V], ov[V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = __ldcs(xr + lane + 32 * i);
    layernorm768_row(v, g, b, eps, ov);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 o = ov[i];
      const int col = (lane + 32 * i) * 4;
      if (y) *reinterpret_cast<float4*>(y + r * ldy + col) = o;
      if (yp) {
        float4 h, l;
        tf32_split(o.x, h.x, l.x);
        tf32_split(o.y, h.y, l.y);
        tf32_split(o.z, h.z, l.z);
        tf32_split(o.w, h.w, l.w);
        *reinterpret_cast<float4*>(yp + r * pld + col) = h;
        *reinterpret_cast<float4*>(yp + pplane + r * pld + col) = l;
      }
      if (yh) {
        __half h0, h1, h2, h3, l0, l1, l2, l3;
        h16_split(o.x, h0, l0);
        h16_split(o.y, h1, l1);
        h16_split(o.z, h2, l2);
        h16_split(o.w, h3, l3);
        *reinterpret_cast<uint2*>(yh + r * hld + col) = make_uint2(pack_h2(h0, h1), pack_h2(h2, h3));
        *reinterpret_cast<uint2*>(yh + hplane + r * hld + col) =
            make_uint2(pack_h2(l0, l1), pack_h2(l2, l3));
      }
    }
  }
}

// The input of a LayerNorm folded into the next GEMM (vit_params.ln_fold): per
// 768-wide row, its FP16 split (planes h16[2][rows][hld]: hi, lo*2^11; a
// magnitude of 32768 or more sets the device error) and, per 32-column slab,
// (sum, M2 about the slab's mean) into stats[slab][rows]. One warp per row:
// lane l holds float4 columns l + 32 i, so slab 4 i + l / 8 lies on eight
// lanes, reduced by three shuffles.
__global__ void __launch_bounds__(256) xsplit_stats768_kernel(
    const float* __restrict__ x, int64_t ldx, int64_t rows, uint16_t* __restrict__ h16,
    int64_t hld, int64_t hplane, float2* __restrict__ stats, int* err) {
  griddep_wait();
  griddep_launch_dependents();
  constexpr int V = 6;
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = warp_global; r < rows; r += nwarps) {
    const float4* xr = reinterpret_cast<const float4*>(x + r * ldx);
    float4 v[V];
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = __ldcs(xr + lane + 32 * i);
    float mx = 0.f, nan = 0.f;  // fmaxf drops NaN; a sum carries it
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 o = v[i];
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(o.x), fabsf(o.y)), fmaxf(fabsf(o.z), fabsf(o.w))));
      float sum = (o.x + o.y) + (o.z + o.w);
      nan += sum - sum;
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      const float mean = sum * (1.f / 32.f);
      const float a0 = o.x - mean, a1 = o.y - mean, a2 = o.z - mean, a3 = o.w - mean;
      float m2 = (a0 * a0 + a1 * a1) + (a2 * a2 + a3 * a3);
      m2 += __shfl_xor_sync(0xffffffffu, m2, 1);
      m2 += __shfl_xor_sync(0xffffffffu, m2, 2);
      m2 += __shfl_xor_sync(0xffffffffu, m2, 4);
      if ((lane & 7) == 0) stats[static_cast<int64_t>(4 * i + lane / 8) * rows + r] = make_float2(sum, m2);
      const int col = (lane + 32 * i) * 4;
      __half h0, h1, h2, h3, l0, l1, l2, l3;
      h16_split(o.x, h0, l0);
      h16_split(o.y, h1, l1);
      h16_split(o.z, h2, l2);
      h16_split(o.w, h3, l3);
      *reinterpret_cast<uint2*>(h16 + r * hld + col) = make_uint2(pack_h2(h0, h1), pack_h2(h2, h3));
      *reinterpret_cast<uint2*>(h16 + hplane + r * hld + col) =
          make_uint2(pack_h2(l0, l1), pack_h2(l2, l3));
    }
    if (!(mx < kH16Limit && nan == 0.f)) report_error(err, kErrF16Range);
  }
}

int xsplit_stats_launch(const float* x, int64_t ldx, int64_t rows, uint16_t* h16, int64_t hld,
                        int64_t hplane, float2* stats, cudaStream_t s) {
  if (rows < 0 || !x || !h16 || !stats) return VITB200_E_INVALID_ARG;
  if (rows == 0) return 0;
  if (reinterpret_cast<uintptr_t>(x) % 16 || ldx % 4 || reinterpret_cast<uintptr_t>(h16) % 8 ||
      hld % 4 || hplane % 4 || reinterpret_cast<uintptr_t>(stats) % 8)
    return VITB200_E_ALIGNMENT;
  int* err = device_error_word();
  if (err == nullptr) return VITB200_E_INVALID_ARG;
  const int threads = 256;
  if (int st_ = launch_kernel(xsplit_stats768_kernel, dim3(grid_for(rows * 32, threads)),
                             dim3(threads), 0, s, 1, x, ldx, rows, h16, hld, hplane, stats, err))
    return st_;
  return cuda_status(cudaGetLastError());
}

// Final LayerNorm of each image's CLS row fused with the classifier head. A
// block serves kHeadImages images and kHeadClasses classes: every warp loads
// its class's head row (the TF32 pair, hi + lo is w to 2^-22) into registers
// while warp w normalises the CLS row of the block's image w into shared
// memory with the LayerNorm kernel's arithmetic (features written out by the
// blocks of the first class group); then each warp takes the FP32 dot products
// y . hi + y . lo plus the bias for the block's images. Every (image, class)
// is computed the same way whatever the batch, so the head is batch invariant.
constexpr int kHeadImages = 8;   // one LayerNorm per warp
constexpr int kHeadClasses = 8;  // one class per warp

__global__ void __launch_bounds__(256) cls_head768_kernel(
    const float* __restrict__ x, int64_t cls_stride, const float* __restrict__ gamma,
    const float* __restrict__ beta, float eps, const float* __restrict__ w_pair,
    const float* __restrict__ bias, int C, int batch, float* __restrict__ logits,
    float* __restrict__ features) {
  griddep_wait();
  griddep_launch_dependents();
  constexpr int E = 768;
  constexpr int V = E / 128;
  __shared__ __align__(16) float4 ys[kHeadImages][E / 4];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int c = blockIdx.x * kHeadClasses + warp;
  const int64_t img0 = static_cast<int64_t>(blockIdx.y) * kHeadImages;
  float4 h[V], l[V];
  if (c < C) {
    const float4* hr = reinterpret_cast<const float4*>(w_pair) + static_cast<int64_t>(c) * (E / 4);
    const float4* lr = reinterpret_cast<const float4*>(w_pair + static_cast<int64_t>(C) * E) +
                       static_cast<int64_t>(c) * (E / 4);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      h[i] = __ldg(hr + lane + 32 * i);
      l[i] = __ldg(lr + lane + 32 * i);
    }
  }
  const int64_t my_img = img0 + warp;
  if (my_img < batch) {
    const float4* xr = reinterpret_cast<const float4*>(x + my_img * cls_stride);
    float4 v[V], g[V], b[V], o[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
      v[i] = __ldg(xr + lane + 32 * i);
      g[i] = __ldg(reinterpret_cast<const float4*>(gamma) + lane + 32 * i);
      b[i] = __ldg(reinterpret_cast<const float4*>(beta) + lane + 32 * i);
    }
    layernorm768_row(v, g, b, eps, o);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      ys[warp][lane + 32 * i] = o[i];
      if (features && blockIdx.x == 0)
        reinterpret_cast<float4*>(features + my_img * E)[lane + 32 * i] = o[i];
    }
  }
  __syncthreads();
  if (c >= C) return;  // uniform across the warp
  const float bc = __ldg(bias + c);
#pragma unroll 1
  for (int k = 0; k < kHeadImages; ++k) {
    const int64_t img = img0 + k;
    if (img >= batch) break;
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 y = ys[k][lane + 32 * i];
      acc = fmaf(y.x, h[i].x, acc);
      acc = fmaf(y.x, l[i].x, acc);
      acc = fmaf(y.y, h[i].y, acc);
      acc = fmaf(y.y, l[i].y, acc);
      acc = fmaf(y.z, h[i].z, acc);
      acc = fmaf(y.z, l[i].z, acc);
      acc = fmaf(y.w, h[i].w, acc);
      acc = fmaf(y.w, l[i].w, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) logits[img * C + c] = acc + bc;
  }
}

int cls_head_launch(const float* x, int64_t cls_stride, const float* gamma, const float* beta,
                    float eps, const float* w_pair, const float* bias, int C, int E, int batch,
                    float* logits, float* features, cudaStream_t s) {
  auto al = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (E != 768 || batch <= 0 || C <= 0 || !x || !gamma || !beta || !w_pair || !bias || !logits ||
      cls_stride % 4 != 0 || !al(x) || !al(gamma) || !al(beta) || !al(w_pair) ||
      (features && !al(features)))
    return VITB200_E_INVALID_ARG;
  const dim3 grid((C + kHeadClasses - 1) / kHeadClasses,
                  (batch + kHeadImages - 1) / kHeadImages);
  if (int st = launch_kernel(cls_head768_kernel, grid, dim3(256), 0, s, 1, x, cls_stride, gamma,
                             beta, eps, w_pair, bias, C, batch, logits, features))
    return st;
  return cuda_status(cudaGetLastError());
}

// Any E: three passes over the row (the re-reads hit L1/L2).
__global__ void layernorm_generic_kernel(const float* __restrict__ x, int64_t ldx,
                                         const float* __restrict__ gamma,
                                         const float* __restrict__ beta, float* __restrict__ y,
                                         int64_t ldy, float* __restrict__ yp, int64_t pld,
                                         int64_t pplane, uint16_t* __restrict__ yh, int64_t hld,
                                         int64_t hplane, int64_t rows, int E, float eps) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = warp_global; r < rows; r += nwarps) {
    const float* xr = x + r * ldx;
    float s = 0.f;
    for (int c = lane; c < E; c += 32) s += xr[c];
    const float mean = warp_sum(s) / static_cast<float>(E);
    float q = 0.f;
    for (int c = lane; c < E; c += 32) {
      const float a = xr[c] - mean;
      q += a * a;
    }
    const float var = warp_sum(q) / static_cast<float>(E);
    const float rstd = 1.0f / sqrtf(var + eps);
    for (int c = lane; c < E; c += 32) {
      const float o = (xr[c] - mean) * rstd * gamma[c] + beta[c];
      if (y) y[r * ldy + c] = o;
      if (yp) {
        float h, l;
        tf32_split(o, h, l);
        yp[r * pld + c] = h;
        yp[pplane + r * pld + c] = l;
      }
      if (yh) {
        __half h, l;
        h16_split(o, h, l);
        yh[r * hld + c] = __half_as_ushort(h);
        yh[hplane + r * hld + c] = __half_as_ushort(l);
      }
    }
  }
}

int layernorm_launch(const float* x, int64_t ldx, const float* gamma, const float* beta,
                     float* y, int64_t ldy, float* y_pair, int64_t pair_ld, int64_t pair_plane,
                     int64_t rows, int E, float eps, cudaStream_t s, uint16_t* y_h16,
                     int64_t h16_ld, int64_t h16_plane) {
  if (rows < 0 || E <= 0 || !x || !gamma || !beta || (!y && !y_pair && !y_h16))
    return VITB200_E_INVALID_ARG;
  if (rows == 0) return 0;
  auto al = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const bool fast = (E == 768) && al(x) && al(gamma) && al(beta) && (ldx % 4 == 0) &&
                    (!y || (al(y) && ldy % 4 == 0)) &&
                    (!y_pair || (al(y_pair) && pair_ld % 4 == 0 && pair_plane % 4 == 0)) &&
                    (!y_h16 || (reinterpret_cast<uintptr_t>(y_h16) % 8 == 0 && h16_ld % 4 == 0 &&
                                h16_plane % 4 == 0));
  const int threads = 256;
  const int64_t work = rows * 32;
  if (fast) {
    if (int st_ = launch_kernel(layernorm768_kernel, dim3(grid_for(work, threads)), dim3(threads),
        0, s, 1, x, ldx, gamma, beta, y, ldy, y_pair, pair_ld, pair_plane, y_h16, h16_ld, h16_plane,
        rows, eps))
      return st_;
  } else {
    if (int st_ = launch_kernel(layernorm_generic_kernel, dim3(grid_for(work, threads)),
        dim3(threads), 0, s, 1, x, ldx, gamma, beta, y, ldy, y_pair, pair_ld, pair_plane, y_h16,
        h16_ld, h16_plane, rows, E, eps))
      return st_;
  }
  return cuda_status(cudaGetLastError());
}

// ----------------------------------------------------------------- im2col
// img[B][C][H][W] -> pair[2][B*P][C*256], patch vector order (c, py, px) and
// patches row-major over the (H/16) x (W/16) grid, as the reference kernel
// csrc/kernels/patch_embed.cu:29-44 and torch's Conv2d weight layout agree.
// With x != null it also writes each image's CLS row of the token matrix,
// x[b][0] = cls + pos[0] (the patch GEMM's epilogue writes rows 1..P). With
// h16 != null the patches are written as FP16 splits instead (planes
// h16[2][B*P][C*256]: hi, lo*2^11; a magnitude reaching the split's limit
// sets the device error).
__global__ void im2col_pair_kernel(const float* __restrict__ img, int B, int C, int H, int W,
                                   float* __restrict__ pair, const float* __restrict__ cls,
                                   const float* __restrict__ pos, float* __restrict__ x, int E,
                                   uint16_t* __restrict__ h16, int* err) {
  griddep_wait();
  griddep_launch_dependents();
  const int gw = W / 16, gh = H / 16;
  const int P = gw * gh;
  const int K = C * 256;
  const int q_per_row = K / 4;
  const int64_t rows = static_cast<int64_t>(B) * P;
  const int64_t total = rows * q_per_row;
  const int64_t plane = rows * K;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / q_per_row;
    const int k = static_cast<int>(i - m * q_per_row) * 4;
    const int64_t b = m / P;
    const int p = static_cast<int>(m - b * P);
    const int gy = p / gw, gx = p - (p / gw) * gw;
    const int c = k >> 8, py = (k >> 4) & 15, px = k & 15;
    const float* src = img + ((b * C + c) * H + gy * 16 + py) * static_cast<int64_t>(W) +
                       gx * 16 + px;
    const float4 v = __ldcs(reinterpret_cast<const float4*>(src));
    if (h16 != nullptr) {
      uint32_t h0, l0, h1, l1;
      h16_split2(v.x, v.y, h0, l0);
      h16_split2(v.z, v.w, h1, l1);
      // fmaxf drops NaN; the sum carries it (and turns inf - inf into NaN).
      const float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
      const float sum = (v.x + v.y) + (v.z + v.w);
      if (!(mx < kH16Limit && sum == sum)) report_error(err, kErrF16Range);
      uint16_t* dst = h16 + m * K + k;
      *reinterpret_cast<uint2*>(dst) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(dst + plane) = make_uint2(l0, l1);
    } else {
      float4 h, l;
      tf32_split(v.x, h.x, l.x);
      tf32_split(v.y, h.y, l.y);
      tf32_split(v.z, h.z, l.z);
      tf32_split(v.w, h.w, l.w);
      float* dst = pair + m * K + k;
      *reinterpret_cast<float4*>(dst) = h;
      *reinterpret_cast<float4*>(dst + plane) = l;
    }
    (void)gh;
  }
  if (x != nullptr) {
    const int64_t T = P + 1;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
         i < static_cast<int64_t>(B) * E; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t b = i / E;
      const int n = static_cast<int>(i - b * E);
      x[b * T * E + n] = cls[n] + pos[n];
    }
  }
}

int im2col_pair_launch(const float* img, int B, int C, int H, int W, float* pair,
                       cudaStream_t s, const float* cls, const float* pos, float* x, int E,
                       uint16_t* h16) {
  if (B < 0 || C <= 0 || H <= 0 || W <= 0 || H % 16 || W % 16 || !img || (!pair && !h16) ||
      (x && (!cls || !pos || E <= 0)))
    return VITB200_E_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(img) % 16 || reinterpret_cast<uintptr_t>(pair) % 16 ||
      reinterpret_cast<uintptr_t>(h16) % 16)
    return VITB200_E_ALIGNMENT;
  if (B == 0) return 0;
  int* err = device_error_word();
  if (err == nullptr) return VITB200_E_INVALID_ARG;
  const int64_t work = static_cast<int64_t>(B) * (H / 16) * (W / 16) * C * 64;
  if (int st_ = launch_kernel(im2col_pair_kernel, dim3(grid_for(work, 256)), dim3(256), 0, s, 1,
      img, B, C, H, W, pair, cls, pos, x, E, h16, err))
    return st_;
  return cuda_status(cudaGetLastError());
}

// ------------------------------------------------------------ CLS + pos
// out[b][0] = cls[b] + pos[0]; when patches != null also
// out[b][1+p] = patches[b][p] + pos[1+p] (csrc/kernels/pos_encoding.cu:8-28 with
// P a runtime value). cls_stride 0 broadcasts one CLS row to every image.
__global__ void cls_pos_kernel(const float* __restrict__ cls, int64_t cls_stride,
                               const float* __restrict__ pos, const float* __restrict__ patches,
                               float* __restrict__ out, int B, int P, int E) {
  griddep_wait();
  griddep_launch_dependents();
  const int T = P + 1;
  const int64_t rows = patches ? static_cast<int64_t>(B) * T : B;
  const int64_t total = rows * E;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / E;
    const int n = static_cast<int>(i - r * E);
    int64_t b, t;
    if (patches) {
      b = r / T;
      t = r - b * T;
    } else {
      b = r;
      t = 0;
    }
    const float base = (t == 0) ? cls[b * cls_stride + n] : patches[(b * P + t - 1) * E + n];
    out[(b * T + t) * E + n] = base + pos[t * E + n];
  }
}

int cls_pos_launch(const float* cls, int64_t cls_stride, const float* pos, const float* patches,
                   float* out, int B, int P, int E, cudaStream_t s) {
  if (B < 0 || P < 0 || E <= 0 || !cls || !pos || !out) return VITB200_E_INVALID_ARG;
  if (B == 0) return 0;
  const int64_t rows = patches ? static_cast<int64_t>(B) * (P + 1) : B;
  if (int st_ = launch_kernel(cls_pos_kernel, dim3(grid_for(rows * E, 256)), dim3(256), 0, s, 1,
      cls, cls_stride, pos, patches, out, B, P, E))
    return st_;
  return cuda_status(cudaGetLastError());
}

// ------------------------------------------------- V transpose + split
// v[B*T][ldv] (head h at columns h*64..h*64+63) -> vt[2][B*heads][64][T4], the
// per-head transposed TF32 pair the attention kernel reads as its V^T operand.
// 32x32 tiles through shared memory keep both the reads and the writes
// coalesced. Keys T..T4-1 are left untouched (the attention's tensor map stops
// at T and zero-fills).
__global__ void split_transpose_v_kernel(const float* __restrict__ v, int64_t ldv, int T,
                                         int heads, int T4, float* __restrict__ vt,
                                         int64_t vt_plane) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float tile[32][33];
  const int bh = blockIdx.z;
  const int b = bh / heads, h = bh - (bh / heads) * heads;
  const int t0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int k = ty; k < 32; k += 8) {
    const int t = t0 + k;
    tile[k][tx] = (t < T) ? v[(static_cast<int64_t>(b) * T + t) * ldv + h * 64 + d0 + tx] : 0.f;
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int t = t0 + tx;
    if (t < T) {
      float hi, lo;
      tf32_split(tile[tx][k], hi, lo);
      const int64_t idx = (static_cast<int64_t>(bh) * 64 + d0 + k) * T4 + t;
      vt[idx] = hi;
      vt[idx + vt_plane] = lo;
    }
  }
}

int split_transpose_v_launch(const float* v, int64_t ldv, int B, int T, int heads, float* vt_pair,
                             cudaStream_t s) {
  if (!v || !vt_pair || B < 0 || T < 0 || heads <= 0 || ldv < heads * 64)
    return VITB200_E_INVALID_ARG;
  if (B == 0 || T == 0) return 0;
  const int T4 = (T + 3) / 4 * 4;
  const int64_t plane = static_cast<int64_t>(B) * heads * 64 * T4;
  dim3 grid((T + 31) / 32, 2, B * heads);
  if (int st_ = launch_kernel(split_transpose_v_kernel, dim3(grid), dim3(dim3(32, 8)), 0, s, 1, v,
      ldv, T, heads, T4, vt_pair, plane))
    return st_;
  return cuda_status(cudaGetLastError());
}

// v[B*T][ldv] * scale -> vt16[2][B*heads][64][T8]: per (image, head) the
// transposed FP16 split planes hi, lo*2^11 (the FP16 attention's V^T operand).
// Same 32x32 shared-memory transpose as the TF32 version.
__global__ void split_transpose_v_f16_kernel(const float* __restrict__ v, int64_t ldv, int T,
                                             int heads, int T8, float scale,
                                             uint16_t* __restrict__ vt, int64_t plane, int* err) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ float tile[32][33];
  const int bh = blockIdx.z;
  const int b = bh / heads, h = bh - (bh / heads) * heads;
  const int t0 = blockIdx.x * 32, d0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int k = ty; k < 32; k += 8) {
    const int t = t0 + k;
    tile[k][tx] = (t < T) ? v[(static_cast<int64_t>(b) * T + t) * ldv + h * 64 + d0 + tx] : 0.f;
  }
  __syncthreads();
  bool bad = false;
  for (int k = ty; k < 32; k += 8) {
    const int t = t0 + tx;
    if (t < T) {
      const float x = __fmul_rn(tile[tx][k], scale);
      bad |= !(fabsf(x) < kH16Limit);
      __half hi, lo;
      h16_split(x, hi, lo);
      const int64_t idx = (static_cast<int64_t>(bh) * 64 + d0 + k) * T8 + t;
      vt[idx] = __half_as_ushort(hi);
      vt[idx + plane] = __half_as_ushort(lo);
    }
  }
  if (bad) report_error(err, kErrF16Range);
}

int split_transpose_v_f16_launch(const float* v, int64_t ldv, int B, int T, int heads, float scale,
                                 uint16_t* vt16, cudaStream_t s) {
  if (!v || !vt16 || B < 0 || T < 0 || heads <= 0 || ldv < heads * 64 || !(scale > 0.f))
    return VITB200_E_INVALID_ARG;
  if (B == 0 || T == 0) return 0;
  int* err = device_error_word();
  if (err == nullptr) return VITB200_E_INVALID_ARG;
  const int T8 = (T + 7) / 8 * 8;
  const int64_t plane = static_cast<int64_t>(B) * heads * 64 * T8;
  dim3 grid((T + 31) / 32, 2, B * heads);
  if (int st_ = launch_kernel(split_transpose_v_f16_kernel, dim3(grid), dim3(dim3(32, 8)), 0, s,
      1, v, ldv, T, heads, T8, scale, vt16, plane, err))
    return st_;
  return cuda_status(cudaGetLastError());
}

// ------------------------------------------------------------ K = 0 GEMM
// With an empty reduction the product is 0; only the epilogue remains
// (bias, GELU, residual), matching the reference CuTe kernel's K=0 behaviour.
__global__ void gemm_k0_kernel(int64_t M, int N, GemmEpilogue e) {
  griddep_wait();
  griddep_launch_dependents();
  const int64_t total = M * N;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t m = i / N;
    const int n = static_cast<int>(i - m * N);
    float v = e.bias ? e.bias[n] : 0.f;
    if (e.gelu) v = gelu_erf(v);
    if (e.residual) v = e.residual[m * e.ldr + n] + v;
    if (e.out) e.out[m * e.ldo + n] = v;
    if (e.out_pair) {
      float h, l;
      tf32_split(v, h, l);
      e.out_pair[m * e.ldp + n] = h;
      e.out_pair[e.pair_plane + m * e.ldp + n] = l;
    }
    if (e.out_h16) {
      __half h, l;
      h16_split(v, h, l);
      e.out_h16[m * e.ldh + n] = __half_as_ushort(h);
      e.out_h16[e.h16_plane + m * e.ldh + n] = __half_as_ushort(l);
    }
  }
}

int gemm_k0_launch(const GemmProblem& p, cudaStream_t s) {
  if (p.epi.mode != kModePlain) return VITB200_E_UNSUPPORTED;
  if (int st_ = launch_kernel(gemm_k0_kernel, dim3(grid_for(p.M * p.N, 256)), dim3(256), 0, s, 1,
      p.M, p.N, p.epi))
    return st_;
  return cuda_status(cudaGetLastError());
}

// ----------------------------------------------------------- diagnostics
// A wait that nothing completes: thread 0 waits on a fresh mbarrier (phase 0
// never completes) with the same bounded helpers the GEMM and attention
// kernels use. After the time limit it records its code in the device error
// word and returns; nothing faults and the context stays usable.
__global__ void wait_timeout_kernel(int* err, int kind) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (kind == 0) {
      (void)mbar_wait(&bar, 0, err, kErrWaitFull);
    } else {
      (void)mbar_wait_acq_cluster(&bar, 0, err, kErrWaitSplit);
    }
  }
}

int wait_timeout_launch(int kind, cudaStream_t s) {
  if (kind != 0 && kind != 1) return VITB200_E_INVALID_ARG;
  int* err = device_error_word();
  if (err == nullptr) return VITB200_E_INVALID_ARG;
  if (int st = launch_kernel(wait_timeout_kernel, dim3(1), dim3(32), 0, s, 1, err, kind)) return st;
  return cuda_status(cudaGetLastError());
}

}  // namespace vitb200
