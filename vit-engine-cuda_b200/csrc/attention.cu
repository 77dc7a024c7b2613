// Non-causal multi-head attention on sm_100a tensor cores, head dim 64, any
// sequence length T, operands given as TF32 hi/lo pairs.
//
// Semantics follow csrc/kernels/attention.cu:20-206 of the reference:
// softmax(Q K^T * scale) V per (image, head), head h in columns h*64..h*64+63 of
// [B*T][ld] rows, keys past T masked, online softmax over key tiles. The
// Blackwell mapping (one CTA per 128 query rows of one (image, head)):
//  * warp 0 (TMA): the Q pair once, then the K pair and the V^T pair of 64-key
//    tiles into a two-stage shared-memory ring (128-byte swizzle; V^T through a
//    4-D map whose key extent is T, so keys past T arrive as zeros);
//  * warp 1 (MMA, one thread): S = Q K^T with tcgen05.mma.kind::tf32 in TF32x3
//    (lo*hi, hi*lo, hi*hi; Q and K K-major in shared memory) into TMEM; then
//    O_j = P V with P read from TMEM as the A operand and V^T (produced
//    transposed per head by the QKV GEMM epilogue) a K-major shared-memory
//    operand, again TF32x3;
//  * warps 2-5 (softmax, one query row per thread): tcgen05.ld of the S row,
//    scale and mask, online max / sum with expf, P written back to TMEM as a
//    TF32 pair (tcgen05.st); then O_j is read back and added into an FP32
//    running output in registers, rescaled by exp(m_old - m_new) — each
//    tensor-core accumulation spans only one 64-key tile, the sum across tiles
//    is round-to-nearest FP32.
// Two TMEM buffer sets let S_{j+1} and O_{j-1} run on the tensor core while the
// softmax warps work on tile j. All waits are bounded (device error word).
#include <math.h>

#include "common.cuh"
#include "engine.h"
#include "vitb200.h"

namespace vitb200 {

namespace {
constexpr int kQ = 128;                       // query rows per CTA
constexpr int kKV = 64;                       // keys per tile
constexpr int kD = 64;                        // head dim
constexpr int kThreadsA = 192;                // TMA, MMA, 4 softmax warps
constexpr int kQBox = 2 * kQ * 32 * 4;        // one 32-column box of the Q pair: hi + lo
constexpr int kQBytes = 2 * kQBox;            // 64 KB
constexpr int kKVBox = 2 * kKV * 32 * 4;      // 16 KB
constexpr int kKBytes = 2 * kKVBox;           // 32 KB (same for V)
constexpr int kStageBytes = 2 * kKBytes;      // K + V = 64 KB
constexpr int kSmem = kQBytes + 2 * kStageBytes + 1024;
constexpr int kSetCols = 3 * kKV;             // S/P_hi | P_lo | O_j
constexpr int kTmemCols = 512;
constexpr uint32_t kIdescS = make_idesc_tf32(kQ, kKV);
constexpr uint32_t kIdescPV = make_idesc_tf32(kQ, kD);  // B = V^T tile, K-major (keys)
}  // namespace

struct AttnArgs {
  int T;
  int n_kv;
  int heads;
  int q_col, k_col;
  float scale;
  float* o;
  int64_t ldo;
  float* o_pair;
  int64_t pld;
  int64_t pplane;
  uint16_t* o_h16;  // FP16 split of O (planes hi | lo * 2^11) or null
  int64_t hld;
  int64_t hplane;
  int* err;
};

__device__ __forceinline__ bool attn_warp_wait(uint64_t* bar, uint32_t parity, int* err,
                                               int code, int lane) {
  int ok = 1;
  if (lane == 0) ok = mbar_wait(bar, parity, err, code) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
}

__device__ __forceinline__ void attn_drain_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t addr = smem_addr(bar);
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(addr, parity)) {
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      report_error(err, kErrDrain);
      return;
    }
  }
}

__global__ void __launch_bounds__(kThreadsA, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmap_q,
                        const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_vt, const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full;
  __shared__ __align__(8) uint64_t kv_full[2];
  __shared__ __align__(8) uint64_t kv_empty[2];
  __shared__ __align__(8) uint64_t s_full[2];
  __shared__ __align__(8) uint64_t p_full[2];
  __shared__ __align__(8) uint64_t pv_full[2];
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = a.err;
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sq = base;
  uint8_t* skv0 = base + kQBytes;

  const int qt = blockIdx.x;
  const int h = blockIdx.y;
  const int row0 = blockIdx.z * a.T;  // first row of this image
  const int q_row = row0 + qt * kQ;
  const int n_kv = a.n_kv;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_full[i], 1);
    }
    mbar_init(&mma_done, 1);
    fence_barrier_init();
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_vt);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  griddep_wait();
  griddep_launch_dependents();

  if (warp == 0) {
    // -------------------------------------------------------------- TMA
    if (lane == 0) {
      mbar_arrive_expect_tx(&q_full, kQBytes);
      tma_load_3d(sq, &tmap_q, &q_full, a.q_col + h * kD, q_row, 0);
      tma_load_3d(sq + kQBox, &tmap_q, &q_full, a.q_col + h * kD + 32, q_row, 0);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int stage = j & 1;
        if (!mbar_wait(&kv_empty[stage], ((j >> 1) & 1) ^ 1, err, kErrWaitEmpty)) break;
        uint8_t* sk = skv0 + stage * kStageBytes;
        uint8_t* sv = sk + kKBytes;
        const int kr = row0 + j * kKV;
        mbar_arrive_expect_tx(&kv_full[stage], kStageBytes);
        tma_load_3d(sk, &tmap_k, &kv_full[stage], a.k_col + h * kD, kr, 0);
        tma_load_3d(sk + kKVBox, &tmap_k, &kv_full[stage], a.k_col + h * kD + 32, kr, 0);
        const int bh = blockIdx.z * a.heads + h;
        tma_load_4d(sv, &tmap_vt, &kv_full[stage], j * kKV, 0, bh, 0);
        tma_load_4d(sv + kKVBox, &tmap_vt, &kv_full[stage], j * kKV + 32, 0, bh, 0);
        ++issued;
      }
      attn_drain_wait(&q_full, 0, err);
      for (int s = 0; s < 2; ++s)
        if (issued > s) attn_drain_wait(&kv_full[s], ((issued - s + 1) / 2 - 1) & 1, err);
    }
  } else if (warp == 1) {
    // -------------------------------------------------------------- MMA
    if (lane == 0) {
      bool ok = mbar_wait(&q_full, 0, err, kErrWaitFull);
      tc_fence_after();
      const uint32_t q_addr = smem_addr(sq);
      auto issue_s = [&](int j) -> bool {
        const int stage = j & 1, set = j & 1;
        if (!mbar_wait(&kv_full[stage], (j >> 1) & 1, err, kErrWaitFull)) return false;
        // S_j overwrites the P of tile j-2 in this set: wait for O_{j-2}.
        if (j >= 2 && !mbar_wait(&pv_full[set], ((j - 2) >> 1) & 1, err, kErrWaitAccEmpty))
          return false;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(set * kSetCols);
        const uint32_t k_addr = smem_addr(skv0 + stage * kStageBytes);
#pragma unroll
        for (int kk = 0; kk < kD / 8; ++kk) {
          const uint32_t off = static_cast<uint32_t>((kk >> 2) * kQBox + (kk & 3) * 32);
          const uint32_t koff = static_cast<uint32_t>((kk >> 2) * kKVBox + (kk & 3) * 32);
          const uint64_t qh = make_sdesc_kmajor(q_addr + off, 128);
          const uint64_t ql = make_sdesc_kmajor(q_addr + off + kQBox / 2, 128);
          const uint64_t kh = make_sdesc_kmajor(k_addr + koff, 128);
          const uint64_t kl = make_sdesc_kmajor(k_addr + koff + kKVBox / 2, 128);
          umma_tf32(d, ql, kh, kIdescS, kk ? 1u : 0u);
          umma_tf32(d, qh, kl, kIdescS, 1u);
          umma_tf32(d, qh, kh, kIdescS, 1u);
        }
        umma_commit(&s_full[set]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int stage = j & 1, set = j & 1;
        if (!mbar_wait(&p_full[set], (j >> 1) & 1, err, kErrWaitAccFull)) return false;
        tc_fence_after();
        const uint32_t p_hi = tmem_base + static_cast<uint32_t>(set * kSetCols);
        const uint32_t p_lo = p_hi + kKV;
        const uint32_t d = p_hi + 2 * kKV;
        const uint32_t v_addr = smem_addr(skv0 + stage * kStageBytes + kKBytes);
#pragma unroll
        for (int kk = 0; kk < kKV / 8; ++kk) {
          const uint32_t voff = static_cast<uint32_t>((kk >> 2) * kKVBox + (kk & 3) * 32);
          const uint64_t vh = make_sdesc_kmajor(v_addr + voff, 128);
          const uint64_t vl = make_sdesc_kmajor(v_addr + voff + kKVBox / 2, 128);
          const uint32_t col = static_cast<uint32_t>(kk * 8);
          umma_tf32_tmem_a(d, p_lo + col, vh, kIdescPV, kk ? 1u : 0u);
          umma_tf32_tmem_a(d, p_hi + col, vl, kIdescPV, 1u);
          umma_tf32_tmem_a(d, p_hi + col, vh, kIdescPV, 1u);
        }
        umma_commit(&pv_full[set]);
        umma_commit(&kv_empty[stage]);  // K_j and V_j are no longer read
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j + 1 < n_kv) ok = issue_s(j + 1);
        if (ok) ok = issue_pv(j);
      }
      umma_commit(&mma_done);
      attn_drain_wait(&mma_done, 0, err);
    }
  } else {
    // -------------------------------------------------------------- softmax
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    float o[kD];
#pragma unroll
    for (int c = 0; c < kD; ++c) o[c] = 0.f;
    float m_run = -INFINITY, l_run = 0.f, alpha_prev = 0.f;
    bool ok = true;

    auto consume_pv = [&](int t, float alpha) -> bool {
      const int set = t & 1;
      if (!attn_warp_wait(&pv_full[set], (t >> 1) & 1, err, kErrWaitAccFull, lane)) return false;
      tc_fence_after();
      const uint32_t col = lane_base + static_cast<uint32_t>(set * kSetCols + 2 * kKV);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float pv[32];
        __syncwarp();
        tmem_ld_32x32b_x32(col + half * 32, pv);
#pragma unroll
        for (int c = 0; c < 32; ++c) o[half * 32 + c] = fmaf(o[half * 32 + c], alpha, pv[c]);
      }
      return true;
    };

    for (int j = 0; j < n_kv; ++j) {
      const int set = j & 1;
      if (!attn_warp_wait(&s_full[set], (j >> 1) & 1, err, kErrWaitAccFull, lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t scol = lane_base + static_cast<uint32_t>(set * kSetCols);
      float s[kKV];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float t[32];
        __syncwarp();
        tmem_ld_32x32b_x32(scol + half * 32, t);
#pragma unroll
        for (int c = 0; c < 32; ++c) s[half * 32 + c] = t[c];
      }
      const int nvalid = min(kKV, a.T - j * kKV);
      float cmax = -INFINITY;
#pragma unroll
      for (int c = 0; c < kKV; ++c) {
        s[c] = (c < nvalid) ? s[c] * a.scale : -INFINITY;
        cmax = fmaxf(cmax, s[c]);
      }
      const float m_new = fmaxf(m_run, cmax);
      const float alpha = expf(m_run - m_new);
      float psum = 0.f;
#pragma unroll
      for (int c = 0; c < kKV; ++c) {
        s[c] = expf(s[c] - m_new);
        psum += s[c];
      }
      l_run = l_run * alpha + psum;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float hi[32], lo[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) tf32_split(s[half * 32 + c], hi[c], lo[c]);
        __syncwarp();
        tmem_st_32x32b_x32(scol + half * 32, hi);
        tmem_st_32x32b_x32(scol + kKV + half * 32, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[set]);
      if (j > 0 && !consume_pv(j - 1, alpha_prev)) {
        ok = false;
        break;
      }
      alpha_prev = alpha;
      m_run = m_new;
    }
    if (ok) ok = consume_pv(n_kv - 1, alpha_prev);
    const int qi = qt * kQ + r;
    if (ok && qi < a.T) {
      const float inv = 1.0f / l_run;
      const int64_t row = static_cast<int64_t>(q_row) + r;
      if (a.o) {
        float* op = a.o + row * a.ldo + h * kD;
#pragma unroll
        for (int c = 0; c < kD; c += 4)
          *reinterpret_cast<float4*>(op + c) =
              make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
      }
      if (a.o_pair) {
        float* ph = a.o_pair + row * a.pld + h * kD;
#pragma unroll
        for (int c = 0; c < kD; c += 4) {
          float4 hv, lv;
          tf32_split(o[c] * inv, hv.x, lv.x);
          tf32_split(o[c + 1] * inv, hv.y, lv.y);
          tf32_split(o[c + 2] * inv, hv.z, lv.z);
          tf32_split(o[c + 3] * inv, hv.w, lv.w);
          *reinterpret_cast<float4*>(ph + c) = hv;
          *reinterpret_cast<float4*>(ph + a.pplane + c) = lv;
        }
      }
      if (a.o_h16) {
        uint16_t* ph = a.o_h16 + row * a.hld + h * kD;
#pragma unroll
        for (int c = 0; c < kD; c += 8) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            __half h0, l0, h1, l1;
            h16_split(o[c + 2 * t] * inv, h0, l0);
            h16_split(o[c + 2 * t + 1] * inv, h1, l1);
            hw[t] = pack_h2(h0, h1);
            lw[t] = pack_h2(l0, l1);
          }
          *reinterpret_cast<uint4*>(ph + c) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
          *reinterpret_cast<uint4*>(ph + a.hplane + c) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

int attention_prepare_device() {
  return cuda_status(
      cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
}

int attention_launch(const float* q_pair, int64_t q_ld, int q_col, const float* k_pair,
                     int64_t k_ld, int k_col, const float* vt_pair, float* o, int64_t ldo,
                     float* o_pair, int64_t pair_ld, int64_t pair_plane, int B, int T, int heads,
                     float scale, cudaStream_t s, uint16_t* o_h16, int64_t h16_ld,
                     int64_t h16_plane) {
  if (B < 0 || T < 0 || heads <= 0 || !q_pair || !k_pair || !vt_pair || (!o && !o_pair && !o_h16))
    return VITB200_E_INVALID_ARG;
  if (B == 0 || T == 0) return 0;
  if (heads > 65535 || B > 65535) return VITB200_E_UNSUPPORTED;
  const int64_t M = static_cast<int64_t>(B) * T;
  if (M > 0x7fffffffLL - kQ || q_ld % 4 || k_ld % 4) return VITB200_E_UNSUPPORTED;
  if (q_col < 0 || k_col < 0 || q_col + heads * kD > q_ld || k_col + heads * kD > k_ld)
    return VITB200_E_INVALID_ARG;
  auto al = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (!al(q_pair) || !al(k_pair) || !al(vt_pair) || (o && (!al(o) || ldo % 4)) ||
      (o_pair && (!al(o_pair) || pair_ld % 4 || pair_plane % 4)) ||
      (o_h16 && (!al(o_h16) || h16_ld % 8 || h16_plane % 8)))
    return VITB200_E_ALIGNMENT;
  CUtensorMap tq, tk, tvt;
  if (int st = make_pair_map(&tq, q_pair, M, static_cast<int>(q_ld), kQ, 32)) return st;
  if (int st = make_pair_map(&tk, k_pair, M, static_cast<int>(k_ld), kKV, 32)) return st;
  {
    // V^T pair [2][B*heads][64][T4]: keys innermost with extent T (zero fill past T).
    const uint64_t T4 = (static_cast<uint64_t>(T) + 3) / 4 * 4;
    const uint64_t bh = static_cast<uint64_t>(B) * heads;
    const uint64_t dims[4] = {static_cast<uint64_t>(T), kD, bh, 2};
    const uint64_t strides[3] = {T4 * 4, kD * T4 * 4, bh * kD * T4 * 4};
    const uint32_t box[4] = {32, kD, 1, 2};
    if (int st = encode_tmap(&tvt, 4, vt_pair, dims, strides, box, 1)) return st;
  }
  AttnArgs a;
  a.T = T;
  a.n_kv = (T + kKV - 1) / kKV;
  a.heads = heads;
  a.q_col = q_col;
  a.k_col = k_col;
  a.scale = scale;
  a.o = o;
  a.ldo = ldo;
  a.o_pair = o_pair;
  a.pld = pair_ld;
  a.pplane = pair_plane;
  a.o_h16 = o_h16;
  a.hld = h16_ld;
  a.hplane = h16_plane;
  a.err = device_error_word();
  dim3 grid((T + kQ - 1) / kQ, heads, B);
  if (int st = launch_kernel(attention_tc_kernel, grid, dim3(kThreadsA), kSmem, s, 1, tq, tk, tvt, a))
    return st;
  return cuda_status(cudaGetLastError());
}

}  // namespace vitb200
