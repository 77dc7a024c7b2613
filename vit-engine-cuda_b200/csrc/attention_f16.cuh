// Shared by the two FP16-split attention kernels (attention_f16.cu: work
// items of two query tiles; attention_f16_tile.cu: one query tile per item,
// for small batches): their launch arguments and small device helpers.
#pragma once

#include <cuda.h>
#include <math.h>

#include "common.cuh"

namespace vitb200 {

struct AttnF16Args {
  int T;
  int n_kv;       // key tiles per item
  int heads;
  int nq;         // query tiles per image
  int qpairs;     // ceil(nq / 2) (two-tile items)
  int n_items;    // work items of the launched kernel
  float s_scale;  // log2(e) * softmax scale / (q_scale * k_scale): S -> log2 units
  float o_scale;  // 1 / v_scale
  float* o;       // fp32 O [M][ldo] or null
  int64_t ldo;
  float* o_pair;  // TF32 pair of O (planes hi | lo) or null
  int64_t pld;
  int64_t pplane;
  uint16_t* o_h16;  // FP16 split of O (planes hi | lo*2^11) or null
  int64_t hld;
  int64_t hplane;
  int* err;
};

// One query tile per item (attention_f16_tile.cu).
int attention_f16_tile_prepare_device();
int attention_f16_tile_launch(const CUtensorMap& tq, const CUtensorMap& tk,
                              const CUtensorMap& tvt, const AttnF16Args& a, cudaStream_t s);

namespace {

__device__ __forceinline__ bool f16_warp_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                              int lane) {
  int ok = 1;
  if (lane == 0) ok = mbar_wait(bar, parity, err, code) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
}

// 2^x for x <= 0 (the hardware approximation, relative error about 2^-22,
// below the FP16 split's own; results under 2^-126 flush to zero, where a
// probability no longer matters against a row maximum of 1).
__device__ __forceinline__ float exp2_nonpos(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void f16_drain_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t addr = smem_addr(bar);
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(addr, parity)) {
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      report_error(err, kErrDrain);
      return;
    }
  }
}

// S = Q K^T for one 128-query x 64-key tile on FP16 splits (descriptors of
// the first 16-wide K slice; a slice further is +2 in the address field): per
// slice the two cross products lo*hi and hi*lo first, then the first hi*hi
// folds them in with scale-input-d (D = A*B + D*2^-11) and the rest follow.
__device__ __forceinline__ void issue_s_f16(uint32_t d, uint64_t qh, uint64_t ql, uint64_t kh,
                                            uint64_t kl, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint64_t o = static_cast<uint64_t>(2 * kk);
    umma_f16(d, ql + o, kh + o, idesc, kk ? 1u : 0u);  // lo * hi
    umma_f16(d, qh + o, kl + o, idesc, 1u);            // hi * lo
  }
  umma_f16_sd11(d, qh, kh, idesc);  // hi * hi + cross * 2^-11
#pragma unroll
  for (int kk = 1; kk < 4; ++kk) {
    const uint64_t o = static_cast<uint64_t>(2 * kk);
    umma_f16(d, qh + o, kh + o, idesc, 1u);            // hi * hi
  }
}

// O_j = P V for one tile with P's FP16 split in TMEM (hi words at p_hi, lo
// at p_lo; two halves per 32-bit column) as the A operand, same product order.
__device__ __forceinline__ void issue_pv_f16(uint32_t d, uint32_t p_hi, uint32_t p_lo, uint64_t vh,
                                             uint64_t vl, uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint64_t o = static_cast<uint64_t>(2 * kk);
    const uint32_t col = static_cast<uint32_t>(kk * 8);
    umma_f16_tmem_a(d, p_lo + col, vh + o, idesc, kk ? 1u : 0u);  // lo * hi
    umma_f16_tmem_a(d, p_hi + col, vl + o, idesc, 1u);            // hi * lo
  }
  umma_f16_tmem_a_sd11(d, p_hi, vh, idesc);  // hi * hi + cross * 2^-11
#pragma unroll
  for (int kk = 1; kk < 4; ++kk) {
    const uint64_t o = static_cast<uint64_t>(2 * kk);
    umma_f16_tmem_a(d, p_hi + kk * 8, vh + o, idesc, 1u);        // hi * hi
  }
}

// One online-softmax step of a query row over a 64-key tile of S (s, raw
// scores; keys from nvalid on are masked), in base 2: exp(x * scale - m) =
// 2^(x * s_scale - m') with m' the running maximum in the same units, one FMA
// rounding each argument. Returns the new running maximum, sets alpha (the
// factor taking the old sums to it), updates l_run and writes P's FP16 split
// (hi words, lo words) into ph, pl. A ragged tile of at most 16 keys (T = 197:
// 5, T = 577: 1; uniform across the warpgroup) runs the arithmetic on 16 keys
// only, the other 48 P entries being zero.
__device__ __forceinline__ float softmax_tile_f16(float (&s)[64], int nvalid, float s_scale,
                                                  float m_run, float& alpha, float& l_run,
                                                  float (&ph)[32], float (&pl)[32]) {
  float m_new;
  if (nvalid <= 16) {
#pragma unroll
    for (int c = 0; c < 16; ++c) s[c] = (c < nvalid) ? s[c] : -INFINITY;
    float cmax = -INFINITY;
#pragma unroll
    for (int c = 0; c < 16; ++c) cmax = fmaxf(cmax, s[c]);
    m_new = fmaxf(m_run, cmax * s_scale);
    alpha = exp2_nonpos(m_run - m_new);
    float psum = 0.f;
#pragma unroll
    for (int c = 0; c < 16; ++c) {
      s[c] = exp2_nonpos(fmaf(s[c], s_scale, -m_new));
      psum += s[c];
    }
    l_run = l_run * alpha + psum;
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      uint32_t hw = 0, lw = 0;
      if (c < 8) h16_split2(s[2 * c], s[2 * c + 1], hw, lw);
      ph[c] = __uint_as_float(hw);
      pl[c] = __uint_as_float(lw);
    }
  } else {
    if (nvalid < 64) {
#pragma unroll
      for (int c = 0; c < 64; ++c) s[c] = (c < nvalid) ? s[c] : -INFINITY;
    }
    float cmax = -INFINITY;
#pragma unroll
    for (int c = 0; c < 64; ++c) cmax = fmaxf(cmax, s[c]);
    m_new = fmaxf(m_run, cmax * s_scale);
    alpha = exp2_nonpos(m_run - m_new);
    float psum = 0.f;
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      s[c] = exp2_nonpos(fmaf(s[c], s_scale, -m_new));
      psum += s[c];
    }
    l_run = l_run * alpha + psum;
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      uint32_t hw, lw;
      h16_split2(s[2 * c], s[2 * c + 1], hw, lw);
      ph[c] = __uint_as_float(hw);
      pl[c] = __uint_as_float(lw);
    }
  }
  return m_new;
}

}  // namespace
}  // namespace vitb200
