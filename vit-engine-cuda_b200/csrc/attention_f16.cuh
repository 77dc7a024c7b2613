// Shared by the two FP16-split attention kernels (attention_f16.cu: work
// items of two query tiles; attention_f16_tile.cu: one query tile per item,
// for small batches): their launch arguments and small device helpers.
#pragma once

#include <cuda.h>

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

}  // namespace
}  // namespace vitb200
