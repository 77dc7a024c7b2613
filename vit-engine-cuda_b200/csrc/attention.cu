// Non-causal multi-head attention, head dim 64, any sequence length T.
//
// Semantics follow csrc/kernels/attention.cu:20-206 of the reference
// (softmax(Q K^T * scale) V per (batch, head); head h in columns h*64..h*64+63
// of [B][T][heads*64] rows; keys past T masked; online softmax), but the
// mapping is different: one CTA owns 128 query rows of one (b, h), each thread
// one query row with its 64-wide q and o in registers; K/V tiles of 64 keys are
// staged in shared memory (read as broadcasts) and consumed in 16-key chunks of
// online softmax with an accurate expf. The output can be written as fp32 and/or
// as the TF32 pair the projection GEMM consumes.
#include <math.h>

#include "common.cuh"
#include "engine.h"
#include "vitb200.h"

namespace vitb200 {

namespace {
constexpr int kD = 64;        // head dim
constexpr int kQ = 128;       // query rows per CTA (one per thread)
constexpr int kKV = 64;       // keys per shared-memory tile
constexpr int kChunk = 16;    // keys per online-softmax update
}  // namespace

__global__ void __launch_bounds__(kQ) attention_simt_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    int64_t ldq, int64_t ldk, int64_t ldv, float* __restrict__ o, int64_t ldo,
    float* __restrict__ o_pair, int64_t pld, int64_t pplane, int T, float scale, int vec_ok) {
  __shared__ float4 sk[kKV][kD / 4];
  __shared__ float4 sv[kKV][kD / 4];

  const int h = blockIdx.y;
  const int64_t b = blockIdx.z;
  const int tid = threadIdx.x;
  const int qi = blockIdx.x * kQ + tid;
  const bool valid = qi < T;
  const int64_t row0 = b * T;

  float qr[kD];
  float acc[kD];
#pragma unroll
  for (int d = 0; d < kD; ++d) acc[d] = 0.f;
  if (valid) {
    const float* qp = q + (row0 + qi) * ldq + h * kD;
#pragma unroll
    for (int d = 0; d < kD; ++d) qr[d] = qp[d];
  } else {
#pragma unroll
    for (int d = 0; d < kD; ++d) qr[d] = 0.f;
  }
  float m_run = -INFINITY;
  float l_run = 0.f;

  for (int j0 = 0; j0 < T; j0 += kKV) {
    __syncthreads();
    // cooperative tile load: kKV rows x 16 float4 for K and for V
    for (int idx = tid; idx < kKV * (kD / 4); idx += kQ) {
      const int r = idx / (kD / 4);
      const int c4 = idx - r * (kD / 4);
      const int j = j0 + r;
      float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
      if (j < T) {
        const float* kp = k + (row0 + j) * ldk + h * kD + c4 * 4;
        const float* vp = v + (row0 + j) * ldv + h * kD + c4 * 4;
        if (vec_ok) {
          kv4 = __ldg(reinterpret_cast<const float4*>(kp));
          vv4 = __ldg(reinterpret_cast<const float4*>(vp));
        } else {
          kv4 = make_float4(kp[0], kp[1], kp[2], kp[3]);
          vv4 = make_float4(vp[0], vp[1], vp[2], vp[3]);
        }
      }
      sk[r][c4] = kv4;
      sv[r][c4] = vv4;
    }
    __syncthreads();
    const int nvalid = min(kKV, T - j0);
    for (int c0 = 0; c0 < nvalid; c0 += kChunk) {
      float s[kChunk];
      float cmax = -INFINITY;
#pragma unroll
      for (int jj = 0; jj < kChunk; ++jj) {
        float dot = 0.f;
#pragma unroll
        for (int d4 = 0; d4 < kD / 4; ++d4) {
          const float4 kk = sk[c0 + jj][d4];
          dot = fmaf(qr[4 * d4 + 0], kk.x, dot);
          dot = fmaf(qr[4 * d4 + 1], kk.y, dot);
          dot = fmaf(qr[4 * d4 + 2], kk.z, dot);
          dot = fmaf(qr[4 * d4 + 3], kk.w, dot);
        }
        dot *= scale;
        if (c0 + jj >= nvalid) dot = -INFINITY;
        s[jj] = dot;
        cmax = fmaxf(cmax, dot);
      }
      const float m_new = fmaxf(m_run, cmax);
      const float corr = expf(m_run - m_new);
      l_run *= corr;
#pragma unroll
      for (int d = 0; d < kD; ++d) acc[d] *= corr;
#pragma unroll
      for (int jj = 0; jj < kChunk; ++jj) {
        const float p = expf(s[jj] - m_new);
        l_run += p;
#pragma unroll
        for (int d4 = 0; d4 < kD / 4; ++d4) {
          const float4 vv = sv[c0 + jj][d4];
          acc[4 * d4 + 0] = fmaf(p, vv.x, acc[4 * d4 + 0]);
          acc[4 * d4 + 1] = fmaf(p, vv.y, acc[4 * d4 + 1]);
          acc[4 * d4 + 2] = fmaf(p, vv.z, acc[4 * d4 + 2]);
          acc[4 * d4 + 3] = fmaf(p, vv.w, acc[4 * d4 + 3]);
        }
      }
      m_run = m_new;
    }
  }

  if (!valid) return;
  const float inv = 1.0f / l_run;
  if (o) {
    float* op = o + (row0 + qi) * ldo + h * kD;
#pragma unroll
    for (int d = 0; d < kD; ++d) op[d] = acc[d] * inv;
  }
  if (o_pair) {
    float* ph = o_pair + (row0 + qi) * pld + h * kD;
#pragma unroll
    for (int d = 0; d < kD; ++d) {
      float hi, lo;
      tf32_split(acc[d] * inv, hi, lo);
      ph[d] = hi;
      ph[pplane + d] = lo;
    }
  }
}

int attention_launch(const float* q, const float* k, const float* v, int64_t ldq, int64_t ldk,
                     int64_t ldv, float* o, int64_t ldo, float* o_pair, int64_t pair_ld,
                     int64_t pair_plane, int B, int T, int heads, float scale, cudaStream_t s) {
  if (B < 0 || T < 0 || heads <= 0 || !q || !k || !v || (!o && !o_pair))
    return VITB200_E_INVALID_ARG;
  if (ldq < heads * kD || ldk < heads * kD || ldv < heads * kD) return VITB200_E_INVALID_ARG;
  if (B == 0 || T == 0) return 0;
  if (heads > 65535 || B > 65535) return VITB200_E_UNSUPPORTED;
  auto al = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const int vec_ok = al(k) && al(v) && ldk % 4 == 0 && ldv % 4 == 0;
  dim3 grid((T + kQ - 1) / kQ, heads, B);
  attention_simt_kernel<<<grid, kQ, 0, s>>>(q, k, v, ldq, ldk, ldv, o, ldo, o_pair, pair_ld,
                                            pair_plane, T, scale, vec_ok);
  count_launch();
  return cuda_status(cudaGetLastError());
}

}  // namespace vitb200
