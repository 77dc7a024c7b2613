// Non-causal multi-head attention on sm_100a tensor cores with FP16-split
// operands: every multiply of S = Q K^T and O = P V is three FP16 tensor-core
// products (hi*hi, hi*lo, lo*hi of x = hi + lo * 2^-11), accumulated in FP32
// per 64-key tile and summed across tiles in FP32 registers. Head dim 64, any
// sequence length T.
//
// Semantics follow csrc/kernels/attention.cu:20-206 of the reference, as the
// TF32 kernel (attention.cu) does: softmax(Q K^T * scale) V per (image, head),
// head h in columns h*64..h*64+63, keys past T masked, online softmax over key
// tiles.
//
// Operands, written by the QKV GEMM epilogue (kModeQKVAttn16):
//   q16  [2][M][E]              hi, lo*2^11 of q * q_scale
//   k16  [2][M][E]              the same two planes of k * k_scale
//   vt16 [2][B*heads][64][T8]   the same two planes of (v * v_scale)^T per
//                               (image, head), T8 = T rounded up to 8
// Per 64-wide tile the two cross products (hi*(lo*2^11), (lo*2^11)*hi) are
// accumulated first, then the first hi*hi product folds them in with
// tcgen05.mma's scale-input-d (D = A*B + D*2^-11) and the rest of hi*hi
// follows: S holds q_scale k_scale (q.k) and O_j v_scale (p.v); the softmax
// and the output undo those powers of two exactly.
//
// Blackwell mapping: persistent CTAs (one per SM) walk work items = (image,
// head, pair of 128-row query tiles), 384 threads:
//  * warp 0 (TMA): an item's Q tiles (loaded once the previous item's last S
//    is issued), then per 64-key tile the K tile and the V^T tile into a
//    four-stage ring; keys past T arrive as zeros (the V^T map's key extent
//    is T);
//  * warp 1 (MMA, one thread): S_g = Q_g K^T for each query tile g into TMEM,
//    then O_g = P_g V with P_g read from TMEM as the A operand;
//  * warpgroups 1 and 2 (softmax of query tile 0 and 1, one row per thread):
//    tcgen05.ld of the S row, scale and mask, online max / sum with expf, P
//    written back to TMEM as its FP16 split (tcgen05.st), then O_j read back
//    and added into the FP32 running output, rescaled by exp(m_old - m_new).
// Two TMEM sets per query tile let S_{j+1} run on the tensor core while the
// softmax works on tile j. The control warpgroup gives registers to the
// softmax warpgroups (setmaxnreg). Every wait is bounded (device error word).
#include <math.h>

#include <algorithm>

#include "attention_f16.cuh"
#include "common.cuh"
#include "engine.h"
#include "vitb200.h"

namespace vitb200 {

namespace {
constexpr int kQ = 128;                          // query rows per tile
constexpr int kKV = 64;                          // keys per tile
constexpr int kD = 64;                           // head dim
constexpr int kQT = 2;                           // query tiles per work item
constexpr int kThreadsF = 384;
constexpr int kQTileBytes = 2 * kQ * kD * 2;     // hi + lo planes: 32 KB
constexpr int kQBufBytes = kQT * kQTileBytes;    // 64 KB
constexpr int kKTileBytes = 2 * kKV * kD * 2;    // 16 KB
constexpr int kVTileBytes = 2 * kD * kKV * 2;    // 16 KB
constexpr int kStageBytesF = kKTileBytes + kVTileBytes;
constexpr int kStagesF = 4;  // K/V ring depth
constexpr int kQBufs = 1;    // Q buffers (the next item's Q loads once the last S is issued)
// Output transpose buffers: per softmax warp 32 rows x 128 B (32 columns of the
// FP16 split at a time: 64 B hi, 64 B lo), 16-byte chunks XOR-swizzled by row.
constexpr int kOutStageBytes = 8 * 32 * 128;
constexpr int kSmemF = kQBufs * kQBufBytes + kStagesF * kStageBytesF + kOutStageBytes + 1024;
constexpr int kPlaneQ = kQ * 128;                // bytes between Q planes (128-byte rows)
constexpr int kPlaneKV = kKV * 128;              // bytes between K / V^T planes
// TMEM: per query tile two sets of [S (64 cols; P's FP16 split overwrites it:
// hi in 32 columns, lo in the next 32) | O_j (64 cols)].
constexpr int kSetColsF = 128;
constexpr int kTileColsF = 2 * kSetColsF;
constexpr int kTmemColsF = 512;
constexpr uint32_t kIdescSF = make_idesc_f16(kQ, kKV);
constexpr uint32_t kIdescPVF = make_idesc_f16(kQ, kD);
// 384 threads launched at 168 registers (65536 / 384); the control warpgroup
// drops to 88 and the softmax warpgroups rise to 208: 128 * 88 + 256 * 208 =
// 384 * 168. build.py checks that ptxas allocated exactly 168.
constexpr uint32_t kCtrlRegsF = 88;
constexpr uint32_t kSoftRegsF = 208;
static_assert(128 * kCtrlRegsF + 256 * kSoftRegsF == 384 * 168, "register split");
static_assert(kSmemF <= 227 * 1024, "shared memory");
}  // namespace

namespace {

struct Item {
  int b, h, qt0, nqt;
};

__device__ __forceinline__ Item decode_item(const AttnF16Args& a, int item) {
  Item it;
  const int per_img = a.heads * a.qpairs;
  it.b = item / per_img;
  const int rem = item - it.b * per_img;
  it.h = rem / a.qpairs;
  const int qp = rem - it.h * a.qpairs;
  it.qt0 = 2 * qp;
  it.nqt = min(kQT, a.nq - it.qt0);
  return it;
}

}  // namespace

__global__ void __launch_bounds__(kThreadsF, 1)
    attention_f16_kernel(const __grid_constant__ CUtensorMap tmap_q,
                         const __grid_constant__ CUtensorMap tmap_k,
                         const __grid_constant__ CUtensorMap tmap_vt, const AttnF16Args a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full[kQBufs];
  __shared__ __align__(8) uint64_t q_empty[kQBufs];
  __shared__ __align__(8) uint64_t kv_full[kStagesF];
  __shared__ __align__(8) uint64_t kv_empty[kStagesF];
  __shared__ __align__(8) uint64_t s_full[kQT][2];
  __shared__ __align__(8) uint64_t p_full[kQT][2];
  __shared__ __align__(8) uint64_t pv_full[kQT][2];
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = a.err;
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sq0 = base;                            // Q buffers
  uint8_t* skv0 = base + kQBufs * kQBufBytes;     // K/V ring
  uint8_t* sout = skv0 + kStagesF * kStageBytesF; // output transpose buffers

  if (threadIdx.x == 0) {
    for (int i = 0; i < kQBufs; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < kStagesF; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int g = 0; g < kQT; ++g)
      for (int i = 0; i < 2; ++i) {
        mbar_init(&s_full[g][i], 1);
        mbar_init(&p_full[g][i], 4);  // one arrival per softmax warp
        mbar_init(&pv_full[g][i], 1);
      }
    mbar_init(&mma_done, 1);
    fence_barrier_init();
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_vt);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, kTmemColsF);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  const int n_kv = a.n_kv;
  griddep_wait();
  griddep_launch_dependents();

  if (warp < 4) {
  setmaxnreg_dec<kCtrlRegsF>();
  if (warp == 0) {
    // ---------------------------------------------------------------- TMA
    if (lane == 0) {
      int local = 0;
      int q_issued = 0;
      int64_t kv_issued = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < a.n_items && ok; item += gridDim.x, ++local) {
        const Item it = decode_item(a, item);
        const int qb = local % kQBufs;
        if (!mbar_wait(&q_empty[qb], static_cast<uint32_t>((local / kQBufs) & 1) ^ 1u, err,
                       kErrWaitEmpty))
          break;
        uint8_t* sq = sq0 + qb * kQBufBytes;
        const int row0 = it.b * a.T;
        ++q_issued;
        mbar_arrive_expect_tx(&q_full[qb], it.nqt * kQTileBytes);
        for (int g = 0; g < it.nqt; ++g)
          tma_load_3d(sq + g * kQTileBytes, &tmap_q, &q_full[qb], it.h * kD,
                      row0 + (it.qt0 + g) * kQ, 0);
        const int bh = it.b * a.heads + it.h;
        for (int j = 0; j < n_kv; ++j) {
          const int64_t t = kv_issued;
          const int st = static_cast<int>(t % kStagesF);
          const uint32_t ph = static_cast<uint32_t>((t / kStagesF) & 1);
          if (!mbar_wait(&kv_empty[st], ph ^ 1u, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sk = skv0 + st * kStageBytesF;
          mbar_arrive_expect_tx(&kv_full[st], kStageBytesF);
          tma_load_3d(sk, &tmap_k, &kv_full[st], it.h * kD, row0 + j * kKV, 0);
          tma_load_4d(sk + kKTileBytes, &tmap_vt, &kv_full[st], j * kKV, 0, bh, 0);
          ++kv_issued;
        }
      }
      // Every copy issued must land before the CTA can exit.
      for (int qb = 0; qb < kQBufs; ++qb)
        if (q_issued > qb) {
          const int fills = (q_issued - qb + kQBufs - 1) / kQBufs;
          f16_drain_wait(&q_full[qb], static_cast<uint32_t>((fills - 1) & 1), err);
        }
      for (int s = 0; s < kStagesF; ++s)
        if (kv_issued > s) {
          const int64_t fills = (kv_issued - s + kStagesF - 1) / kStagesF;
          f16_drain_wait(&kv_full[s], static_cast<uint32_t>((fills - 1) & 1), err);
        }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA
    if (lane == 0) {
      int local = 0;
      int64_t kv_used = 0;   // key tiles consumed so far (ring position)
      int64_t tc[kQT] = {0, 0};  // S/P/PV tiles per query tile so far (TMEM set position)
      bool ok = true;
      for (int item = blockIdx.x; item < a.n_items && ok; item += gridDim.x, ++local) {
        const Item it = decode_item(a, item);
        const int qb = local % kQBufs;
        if (!mbar_wait(&q_full[qb], static_cast<uint32_t>((local / kQBufs) & 1), err,
                       kErrWaitFull))
          break;
        tc_fence_after();
        const uint32_t q_addr = smem_addr(sq0 + qb * kQBufBytes);
        auto issue_s = [&](int j) -> bool {
          const int64_t t = kv_used + j;
          const int st = static_cast<int>(t % kStagesF);
          if (!mbar_wait(&kv_full[st], static_cast<uint32_t>((t / kStagesF) & 1), err,
                         kErrWaitFull))
            return false;
          tc_fence_after();
          const uint32_t k_addr = smem_addr(skv0 + st * kStageBytesF);
          for (int g = 0; g < it.nqt; ++g) {
            const int64_t tg = tc[g] + j;
            const int set = static_cast<int>(tg & 1);
            // S overwrites the P of this set's previous tile: wait for its PV.
            if (tg >= 2 &&
                !mbar_wait(&pv_full[g][set], static_cast<uint32_t>(((tg - 2) >> 1) & 1), err,
                           kErrWaitAccEmpty))
              return false;
            tc_fence_after();
            const uint32_t d = tmem_base + static_cast<uint32_t>(g * kTileColsF + set * kSetColsF);
            const uint32_t qa = q_addr + g * kQTileBytes;
            // Descriptors of slice 0; a 16-wide K slice further is +32 bytes,
            // i.e. +2 in the descriptor's address field.
            const uint64_t qh = make_sdesc_kmajor(qa, 128);
            const uint64_t ql = make_sdesc_kmajor(qa + kPlaneQ, 128);
            const uint64_t kh = make_sdesc_kmajor(k_addr, 128);
            const uint64_t kl = make_sdesc_kmajor(k_addr + kPlaneKV, 128);
            issue_s_f16(d, qh, ql, kh, kl, kIdescSF);
            umma_commit(&s_full[g][set]);
          }
          return true;
        };
        auto issue_pv = [&](int j) -> bool {
          const int64_t t = kv_used + j;
          const int st = static_cast<int>(t % kStagesF);
          const uint32_t v_addr = smem_addr(skv0 + st * kStageBytesF + kKTileBytes);
          for (int g = 0; g < it.nqt; ++g) {
            const int64_t tg = tc[g] + j;
            const int set = static_cast<int>(tg & 1);
            if (!mbar_wait(&p_full[g][set], static_cast<uint32_t>((tg >> 1) & 1), err,
                           kErrWaitAccFull))
              return false;
            tc_fence_after();
            const uint32_t p_hi =
                tmem_base + static_cast<uint32_t>(g * kTileColsF + set * kSetColsF);
            const uint32_t p_lo = p_hi + 32;
            const uint32_t d = p_hi + 64;
            const uint64_t vh = make_sdesc_kmajor(v_addr, 128);
            const uint64_t vl = make_sdesc_kmajor(v_addr + kPlaneKV, 128);
            issue_pv_f16(d, p_hi, p_lo, vh, vl, kIdescPVF);
            umma_commit(&pv_full[g][set]);
          }
          umma_commit(&kv_empty[st]);  // K_j and V_j are no longer read
          return true;
        };
        ok = issue_s(0);
        if (ok && n_kv == 1) umma_commit(&q_empty[qb]);
        for (int j = 0; ok && j < n_kv; ++j) {
          if (j + 1 < n_kv) {
            ok = issue_s(j + 1);
            if (ok && j + 2 == n_kv) umma_commit(&q_empty[qb]);  // last S of the item
          }
          if (ok) ok = issue_pv(j);
        }
        kv_used += n_kv;
        for (int g = 0; g < it.nqt; ++g) tc[g] += n_kv;
      }
      // Every MMA issued must finish before TMEM is released.
      umma_commit(&mma_done);
      f16_drain_wait(&mma_done, 0, err);
    }
  }
  } else {
    setmaxnreg_inc<kSoftRegsF>();
    // ------------------------------------------------------------ softmax
    const int g = (warp - 4) >> 2;  // query tile of this warpgroup
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                               static_cast<uint32_t>(g * kTileColsF);
    int64_t tcount = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < a.n_items && ok; item += gridDim.x) {
      const Item it = decode_item(a, item);
      if (g >= it.nqt) continue;
      float o[kD];
#pragma unroll
      for (int c = 0; c < kD; ++c) o[c] = 0.f;
      float m_run = -INFINITY, l_run = 0.f, alpha_prev = 0.f;

      auto consume_pv = [&](int64_t t, float alpha) -> bool {
        const int set = static_cast<int>(t & 1);
        if (!f16_warp_wait(&pv_full[g][set], static_cast<uint32_t>((t >> 1) & 1), err,
                           kErrWaitAccFull, lane))
          return false;
        tc_fence_after();
        const uint32_t col = lane_base + static_cast<uint32_t>(set * kSetColsF + 64);
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
        const int64_t t = tcount + j;
        const int set = static_cast<int>(t & 1);
        if (!f16_warp_wait(&s_full[g][set], static_cast<uint32_t>((t >> 1) & 1), err,
                           kErrWaitAccFull, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t scol = lane_base + static_cast<uint32_t>(set * kSetColsF);
        float s[kKV];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float tt[32];
          __syncwarp();
          tmem_ld_32x32b_x32(scol + half * 32, tt);
#pragma unroll
          for (int c = 0; c < 32; ++c) s[half * 32 + c] = tt[c];
        }
        // P_t (and the running max / sum) from this tile's scores.
        const int nvalid = a.T - j * kKV;
        float alpha;
        float ph[32], pl[32];
        const float m_new = softmax_tile_f16(s, nvalid, a.s_scale, m_run, alpha, l_run, ph, pl);
        __syncwarp();
        tmem_st_32x32b_x32(scol, ph);
        tmem_st_32x32b_x32(scol + 32, pl);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g][set]);
        if (j > 0 && !consume_pv(t - 1, alpha_prev)) {
          ok = false;
          break;
        }
        alpha_prev = alpha;
        m_run = m_new;
      }
      if (ok) ok = consume_pv(tcount + n_kv - 1, alpha_prev);
      tcount += n_kv;
      const int qi = (it.qt0 + g) * kQ + r;
      if (ok && qi < a.T) {
        const float inv = a.o_scale / l_run;
        const int64_t row = static_cast<int64_t>(it.b) * a.T + qi;
        if (a.o) {
          float* op = a.o + row * a.ldo + it.h * kD;
#pragma unroll
          for (int c = 0; c < kD; c += 4)
            *reinterpret_cast<float4*>(op + c) =
                make_float4(o[c] * inv, o[c + 1] * inv, o[c + 2] * inv, o[c + 3] * inv);
        }
        if (a.o_pair) {
          float* pp = a.o_pair + row * a.pld + it.h * kD;
#pragma unroll
          for (int c = 0; c < kD; c += 4) {
            float4 hv, lv;
            tf32_split(o[c] * inv, hv.x, lv.x);
            tf32_split(o[c + 1] * inv, hv.y, lv.y);
            tf32_split(o[c + 2] * inv, hv.z, lv.z);
            tf32_split(o[c + 3] * inv, hv.w, lv.w);
            *reinterpret_cast<float4*>(pp + c) = hv;
            *reinterpret_cast<float4*>(pp + a.pplane + c) = lv;
          }
        }
      }
      if (ok && a.o_h16) {
        // FP16 split of O through the warp's transpose buffer, 32 columns at a
        // time, so that each store instruction writes four whole 64-byte row
        // segments (lanes 0-3 of each eight: hi, lanes 4-7: lo).
        const float inv = a.o_scale / l_run;  // rows past T are computed, not stored
        uint32_t* stg = reinterpret_cast<uint32_t*>(sout) + (warp - 4) * 32 * 32;
        const int first = (it.qt0 + g) * kQ + quarter * 32;  // token of lane 0's row
        const int valid = a.T - first;
        const int64_t row0 = static_cast<int64_t>(it.b) * a.T + first;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int c = half * 32 + 8 * k + 2 * u;
              h16_split2(o[c] * inv, o[c + 1] * inv, hw[u], lw[u]);
            }
            *reinterpret_cast<uint4*>(stg + lane * 32 + 4 * (k ^ (lane & 7))) =
                make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(stg + lane * 32 + 4 * ((4 + k) ^ (lane & 7))) =
                make_uint4(lw[0], lw[1], lw[2], lw[3]);
          }
          __syncwarp();
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int rr = 4 * q + (lane >> 3);
            const int c = lane & 7;
            const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * 32 + 4 * (c ^ (rr & 7)));
            if (rr < valid)
              *reinterpret_cast<uint4*>(a.o_h16 + (c >> 2) * a.hplane + (row0 + rr) * a.hld +
                                        it.h * kD + half * 32 + (c & 3) * 8) = v;
          }
          __syncwarp();
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemColsF);
  }
}

int attention_f16_prepare_device() {
  if (int st = cuda_status(cudaFuncSetAttribute(
          attention_f16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemF)))
    return st;
  return attention_f16_tile_prepare_device();
}

int attention_f16_launch(const uint16_t* q16, const uint16_t* k16, int64_t ld, const uint16_t* vt16,
                         int T8, float* o, int64_t ldo, float* o_pair, int64_t pair_ld,
                         int64_t pair_plane, uint16_t* o_h16, int64_t h16_ld, int64_t h16_plane,
                         int B, int T, int heads, float scale, float q_scale, float k_scale,
                         float v_scale, cudaStream_t s) {
  if (B < 0 || T < 0 || heads <= 0 || !q16 || !k16 || !vt16 || (!o && !o_pair && !o_h16))
    return VITB200_E_INVALID_ARG;
  if (!(q_scale > 0.f) || !(k_scale > 0.f) || !(v_scale > 0.f)) return VITB200_E_INVALID_ARG;
  if (B == 0 || T == 0) return 0;
  if (ld < static_cast<int64_t>(heads) * kD || ld % 8 || T8 < T || T8 % 8)
    return VITB200_E_INVALID_ARG;
  const int64_t M = static_cast<int64_t>(B) * T;
  if (M > 0x7fffffffLL - kQ) return VITB200_E_UNSUPPORTED;
  auto al = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (!al(q16) || !al(k16) || !al(vt16) || (o && (!al(o) || ldo % 4)) ||
      (o_pair && (!al(o_pair) || pair_ld % 4 || pair_plane % 4)) ||
      (o_h16 && (!al(o_h16) || h16_ld % 8 || h16_plane % 8)))
    return VITB200_E_ALIGNMENT;
  CUtensorMap tq, tk, tvt;
  if (int st = make_planes_map(&tq, q16, M, static_cast<int>(ld), 2, kQ, kD, 1)) return st;
  if (int st = make_planes_map(&tk, k16, M, static_cast<int>(ld), 2, kKV, kD, 1)) return st;
  {
    // V^T [2][B*heads][64][T8]: keys innermost with extent T (zero fill past T).
    const uint64_t bh = static_cast<uint64_t>(B) * heads;
    const uint64_t t8 = static_cast<uint64_t>(T8);
    const uint64_t dims[4] = {static_cast<uint64_t>(T), kD, bh, 2};
    const uint64_t strides[3] = {t8 * 2, kD * t8 * 2, bh * kD * t8 * 2};
    const uint32_t box[4] = {kKV, kD, 1, 2};
    if (int st = encode_tmap_typed(&tvt, 4, vt16, dims, strides, box, 1, 1)) return st;
  }
  AttnF16Args a;
  a.T = T;
  a.n_kv = (T + kKV - 1) / kKV;
  a.heads = heads;
  a.nq = (T + kQ - 1) / kQ;
  a.qpairs = (a.nq + kQT - 1) / kQT;
  const int64_t items = static_cast<int64_t>(B) * heads * a.qpairs;
  if (items > 0x7fffffffLL) return VITB200_E_UNSUPPORTED;
  a.n_items = static_cast<int>(items);
  a.s_scale = 1.4426950408889634f * scale / (q_scale * k_scale);
  a.o_scale = 1.f / v_scale;
  a.o = o;
  a.ldo = ldo;
  a.o_pair = o_pair;
  a.pld = pair_ld;
  a.pplane = pair_plane;
  a.o_h16 = o_h16;
  a.hld = h16_ld;
  a.hplane = h16_plane;
  a.err = device_error_word();
  if (a.err == nullptr) return VITB200_E_INVALID_ARG;
  // Small batches (two-tile items filling under half the SMs, e.g. batch 1:
  // 12 items): one query tile per item instead (attention_f16_tile.cu).
  if (2 * items < device_num_sms()) {
    a.n_items = static_cast<int>(static_cast<int64_t>(B) * heads * a.nq);
    return attention_f16_tile_launch(tq, tk, tvt, a, s);
  }
  const int grid = static_cast<int>(std::min<int64_t>(items, device_num_sms()));
  if (int st = launch_kernel(attention_f16_kernel, dim3(grid), dim3(kThreadsF), kSmemF, s, 1, tq, tk,
                             tvt, a))
    return st;
  return cuda_status(cudaGetLastError());
}

}  // namespace vitb200
