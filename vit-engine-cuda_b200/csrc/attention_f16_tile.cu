// FP16-split attention with one 128-row query tile per work item, for small
// batches (the two-tile kernel in attention_f16.cu would leave most SMs
// idle there: batch 1 has 12 of its items). Same operands, arithmetic and
// outputs as that kernel (see its header for the FP16-split scheme); the
// difference is the schedule:
//  * work items = (image, head, query tile);
//  * TMEM holds four sets of [S | O_j]; key tile t (counted across items) uses
//    set t % 4, so S runs up to three tiles ahead of PV (a four-stage K/V ring);
//  * softmax warpgroup w takes the key tiles with t % 2 == w for all 128 rows
//    (a set always returns to the same warpgroup), each with its own running
//    max, sum and output; at the end of an item the two exchange their
//    partials through shared memory (bounded mbarrier waits) and each
//    normalises and stores 32 of the 64 output columns.
// Every wait is bounded (device error word).
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
constexpr int kThreadsF = 384;
constexpr int kQTileBytes = 2 * kQ * kD * 2;     // hi + lo planes: 32 KB
constexpr int kKTileBytes = 2 * kKV * kD * 2;    // 16 KB
constexpr int kVTileBytes = 2 * kD * kKV * 2;    // 16 KB
constexpr int kStageBytesF = kKTileBytes + kVTileBytes;
constexpr int kStagesF = 4;  // K/V ring depth (S runs up to three tiles ahead of PV)
constexpr int kSets = 4;     // TMEM sets: key tile t (counted across items) uses set t % 4
// End of an item: the two softmax warpgroups exchange their partial results,
// per warpgroup [34][128] floats (32 O columns, the running max and sum; one
// row per thread, so a warp's accesses are contiguous). The same bytes then
// hold the output transpose buffers: per softmax warp 32 rows x 128 B (32
// columns of the FP16 split: 64 B hi, 64 B lo), 16-byte chunks XOR-swizzled by
// row, warpgroup w's four inside its own exchange half.
constexpr int kXchgFloats = 34 * kQ;
constexpr int kXchgBytes = 2 * kXchgFloats * 4;
constexpr int kOutWarpBytes = 32 * 128;
static_assert(4 * kOutWarpBytes <= kXchgFloats * 4, "output buffers fit an exchange half");
constexpr int kSmemF = kQTileBytes + kStagesF * kStageBytesF + kXchgBytes + 1024;
constexpr int kPlaneQ = kQ * 128;                // bytes between Q planes (128-byte rows)
constexpr int kPlaneKV = kKV * 128;              // bytes between K / V^T planes
// TMEM: four sets of [S (64 cols; P's FP16 split overwrites it: hi in 32
// columns, lo in the next 32) | O_j (64 cols)].
constexpr int kSetColsF = 128;
constexpr int kTmemColsF = kSets * kSetColsF;
constexpr uint32_t kIdescSF = make_idesc_f16(kQ, kKV);
constexpr uint32_t kIdescPVF = make_idesc_f16(kQ, kD);
// 384 threads launched at 168 registers (65536 / 384); the control warpgroup
// drops to 88 and the softmax warpgroups rise to 208: 128 * 88 + 256 * 208 =
// 384 * 168. build.py checks that ptxas allocated exactly 168.
constexpr uint32_t kCtrlRegsF = 88;
constexpr uint32_t kSoftRegsF = 208;
static_assert(128 * kCtrlRegsF + 256 * kSoftRegsF == 384 * 168, "register split");
static_assert(kSmemF <= 227 * 1024, "shared memory");
static_assert(kTmemColsF == 512, "TMEM columns");
}  // namespace

namespace {

struct Item {
  int b, h, qt;
};

// Items in (image, head, query tile) order: the query tiles of one head run
// on neighbouring CTAs and share its K and V tiles in L2.
__device__ __forceinline__ Item decode_item(const AttnF16Args& a, int item) {
  Item it;
  const int per_img = a.heads * a.nq;
  it.b = item / per_img;
  const int rem = item - it.b * per_img;
  it.h = rem / a.nq;
  it.qt = rem - it.h * a.nq;
  return it;
}

}  // namespace

__global__ void __launch_bounds__(kThreadsF, 1)
    attention_f16_tile_kernel(const __grid_constant__ CUtensorMap tmap_q,
                         const __grid_constant__ CUtensorMap tmap_k,
                         const __grid_constant__ CUtensorMap tmap_vt, const AttnF16Args a) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t q_full;
  __shared__ __align__(8) uint64_t q_empty;
  __shared__ __align__(8) uint64_t kv_full[kStagesF];
  __shared__ __align__(8) uint64_t kv_empty[kStagesF];
  __shared__ __align__(8) uint64_t s_full[kSets];
  __shared__ __align__(8) uint64_t p_full[kSets];
  __shared__ __align__(8) uint64_t pv_full[kSets];
  __shared__ __align__(8) uint64_t xchg_bar[2];  // the softmax warpgroups' exchange, per item
  __shared__ __align__(8) uint64_t mma_done;
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = a.err;
  const uint32_t raw = smem_addr(smem_raw);
  uint8_t* base = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint8_t* sq0 = base;                            // Q tile
  uint8_t* skv0 = base + kQTileBytes;             // K/V ring
  float* xchg = reinterpret_cast<float*>(skv0 + kStagesF * kStageBytesF);  // exchange / output

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    for (int i = 0; i < kStagesF; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < kSets; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);  // one arrival per warp of the owning softmax warpgroup
      mbar_init(&pv_full[i], 1);
    }
    mbar_init(&xchg_bar[0], 8);  // one arrival per softmax warp
    mbar_init(&xchg_bar[1], 8);
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
      int64_t kv_issued = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < a.n_items && ok; item += gridDim.x, ++local) {
        const Item it = decode_item(a, item);
        if (!mbar_wait(&q_empty, static_cast<uint32_t>(local & 1) ^ 1u, err, kErrWaitEmpty))
          break;
        const int row0 = it.b * a.T;
        mbar_arrive_expect_tx(&q_full, kQTileBytes);
        tma_load_3d(sq0, &tmap_q, &q_full, it.h * kD, row0 + it.qt * kQ, 0);
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
      if (local > 0) f16_drain_wait(&q_full, static_cast<uint32_t>((local - 1) & 1), err);
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
      int64_t t0 = 0;  // key tiles of earlier items (ring position, TMEM set)
      bool ok = true;
      for (int item = blockIdx.x; item < a.n_items && ok; item += gridDim.x, ++local) {
        if (!mbar_wait(&q_full, static_cast<uint32_t>(local & 1), err, kErrWaitFull)) break;
        tc_fence_after();
        const uint32_t q_addr = smem_addr(sq0);
        const uint64_t qh = make_sdesc_kmajor(q_addr, 128);
        const uint64_t ql = make_sdesc_kmajor(q_addr + kPlaneQ, 128);
        // S_t = Q K_t^T into set t % 4, once that set's previous P has been
        // read by its PV (tile t - 4).
        auto issue_s = [&](int j) -> bool {
          const int64_t t = t0 + j;
          const int st = static_cast<int>(t % kStagesF);
          if (!mbar_wait(&kv_full[st], static_cast<uint32_t>((t / kStagesF) & 1), err,
                         kErrWaitFull))
            return false;
          const int set = static_cast<int>(t & (kSets - 1));
          if (t >= kSets &&
              !mbar_wait(&pv_full[set], static_cast<uint32_t>(((t - kSets) / kSets) & 1), err,
                         kErrWaitAccEmpty))
            return false;
          tc_fence_after();
          const uint32_t k_addr = smem_addr(skv0 + st * kStageBytesF);
          const uint32_t d = tmem_base + static_cast<uint32_t>(set * kSetColsF);
          // Descriptors of slice 0; a 16-wide K slice further is +32 bytes,
          // i.e. +2 in the descriptor's address field.
          const uint64_t kh = make_sdesc_kmajor(k_addr, 128);
          const uint64_t kl = make_sdesc_kmajor(k_addr + kPlaneKV, 128);
          issue_s_f16(d, qh, ql, kh, kl, kIdescSF);
          umma_commit(&s_full[set]);
          return true;
        };
        // O_t = P_t V_t into the set's O columns, once the softmax has written P_t.
        auto issue_pv = [&](int j) -> bool {
          const int64_t t = t0 + j;
          const int st = static_cast<int>(t % kStagesF);
          const int set = static_cast<int>(t & (kSets - 1));
          if (!mbar_wait(&p_full[set], static_cast<uint32_t>((t / kSets) & 1), err,
                         kErrWaitAccFull))
            return false;
          tc_fence_after();
          const uint32_t v_addr = smem_addr(skv0 + st * kStageBytesF + kKTileBytes);
          const uint32_t p_hi = tmem_base + static_cast<uint32_t>(set * kSetColsF);
          const uint32_t p_lo = p_hi + 32;
          const uint32_t d = p_hi + 64;
          const uint64_t vh = make_sdesc_kmajor(v_addr, 128);
          const uint64_t vl = make_sdesc_kmajor(v_addr + kPlaneKV, 128);
          issue_pv_f16(d, p_hi, p_lo, vh, vl, kIdescPVF);
          umma_commit(&pv_full[set]);
          umma_commit(&kv_empty[st]);  // K_t and V_t are no longer read
          return true;
        };
        // S runs up to three tiles ahead of PV (four sets).
        int next_s = 0;
        for (int j = 0; ok && j < n_kv; ++j) {
          while (ok && next_s < n_kv && next_s <= j + kSets - 1) {
            ok = issue_s(next_s++);
            if (ok && next_s == n_kv) umma_commit(&q_empty);  // the item's last S
          }
          if (ok) ok = issue_pv(j);
        }
        t0 += n_kv;
      }
      // Every MMA issued must finish before TMEM is released.
      umma_commit(&mma_done);
      f16_drain_wait(&mma_done, 0, err);
    }
  }
  } else {
    setmaxnreg_inc<kSoftRegsF>();
    // ------------------------------------------------------------ softmax
    // Warpgroup w takes the key tiles t with t % 2 == w (t counted across
    // items, so a TMEM set always returns to the same warpgroup) for all 128
    // query rows, one row per thread, with its own running max, sum and output.
    const int wg = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    int64_t t0 = 0;
    bool ok = true;
    // Both softmax warpgroups at the same point of an item (a bounded wait, so
    // that a warpgroup that gave up on an earlier wait cannot stall the other).
    auto groups_sync = [&](int which, int local) -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(&xchg_bar[which]);
      const bool got = f16_warp_wait(&xchg_bar[which], static_cast<uint32_t>(local & 1), err,
                                     kErrWaitAccFull, lane);
      __syncwarp();
      return got;
    };
    int local = 0;
    for (int item = blockIdx.x; item < a.n_items && ok; item += gridDim.x, ++local) {
      const Item it = decode_item(a, item);
      float o[kD];
#pragma unroll
      for (int c = 0; c < kD; ++c) o[c] = 0.f;
      float m_run = -INFINITY, l_run = 0.f, alpha_prev = 0.f;

      auto consume_pv = [&](int64_t t, float alpha) -> bool {
        const int set = static_cast<int>(t & (kSets - 1));
        if (!f16_warp_wait(&pv_full[set], static_cast<uint32_t>((t / kSets) & 1), err,
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

      int64_t prev = -1;  // this warpgroup's previous tile of the item
      for (int j = 0; j < n_kv; ++j) {
        const int64_t t = t0 + j;
        if (static_cast<int>(t & 1) != wg) continue;
        const int set = static_cast<int>(t & (kSets - 1));
        if (!f16_warp_wait(&s_full[set], static_cast<uint32_t>((t / kSets) & 1), err,
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
        if (lane == 0) mbar_arrive(&p_full[set]);
        // O of this warpgroup's previous tile, rescaled to that tile's max.
        if (prev >= 0 && !consume_pv(prev, alpha_prev)) {
          ok = false;
          break;
        }
        prev = t;
        alpha_prev = alpha;
        m_run = m_new;
      }
      if (ok && prev >= 0) ok = consume_pv(prev, alpha_prev);
      t0 += n_kv;
      if (!ok) break;

      // Combine the two warpgroups' partials (a warpgroup without tiles in
      // this item has m = -inf, l = 0, o = 0): each hands the other the 32
      // output columns the other writes, then writes its own 32 columns.
      float* mine = xchg + wg * kXchgFloats;
      const float* theirs = xchg + (1 - wg) * kXchgFloats;
      // (static register indices: o stays in registers)
#pragma unroll
      for (int c = 0; c < 32; ++c) mine[c * kQ + r] = wg == 0 ? o[32 + c] : o[c];
      mine[32 * kQ + r] = m_run;
      mine[33 * kQ + r] = l_run;
      if (!groups_sync(0, local)) {
        ok = false;
        break;
      }
      const float m_other = theirs[32 * kQ + r];
      const float l_other = theirs[33 * kQ + r];
      const float m_all = fmaxf(m_run, m_other);  // finite: some tile has a valid key
      const float f_mine = exp2_nonpos(m_run - m_all);
      const float f_other = exp2_nonpos(m_other - m_all);
      float oc[32];
#pragma unroll
      for (int c = 0; c < 32; ++c)
        oc[c] = fmaf(wg == 0 ? o[c] : o[32 + c], f_mine, theirs[c * kQ + r] * f_other);
      const float l_all = fmaf(l_run, f_mine, l_other * f_other);
      if (!groups_sync(1, local)) {  // both read before the bytes become output buffers
        ok = false;
        break;
      }

      const int col0 = it.h * kD + wg * 32;  // this warpgroup's output columns
      const int qi = it.qt * kQ + r;
      const float inv = a.o_scale / l_all;
      if (qi < a.T) {
        const int64_t row = static_cast<int64_t>(it.b) * a.T + qi;
        if (a.o) {
          float* op = a.o + row * a.ldo + col0;
#pragma unroll
          for (int c = 0; c < 32; c += 4)
            *reinterpret_cast<float4*>(op + c) =
                make_float4(oc[c] * inv, oc[c + 1] * inv, oc[c + 2] * inv, oc[c + 3] * inv);
        }
        if (a.o_pair) {
          float* pp = a.o_pair + row * a.pld + col0;
#pragma unroll
          for (int c = 0; c < 32; c += 4) {
            float4 hv, lv;
            tf32_split(oc[c] * inv, hv.x, lv.x);
            tf32_split(oc[c + 1] * inv, hv.y, lv.y);
            tf32_split(oc[c + 2] * inv, hv.z, lv.z);
            tf32_split(oc[c + 3] * inv, hv.w, lv.w);
            *reinterpret_cast<float4*>(pp + c) = hv;
            *reinterpret_cast<float4*>(pp + a.pplane + c) = lv;
          }
        }
      }
      if (a.o_h16) {
        // FP16 split of the warpgroup's 32 columns through the warp's
        // transpose buffer, so that each store instruction writes four whole
        // 64-byte row segments (lanes 0-3 of each eight: hi, lanes 4-7: lo).
        // Rows past T are computed, not stored.
        uint32_t* stg = reinterpret_cast<uint32_t*>(mine) + quarter * (kOutWarpBytes / 4);
        const int first = it.qt * kQ + quarter * 32;  // token of lane 0's row
        const int valid = a.T - first;
        const int64_t row0 = static_cast<int64_t>(it.b) * a.T + first;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint32_t hw[4], lw[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int c = 8 * k + 2 * u;
            h16_split2(oc[c] * inv, oc[c + 1] * inv, hw[u], lw[u]);
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
                                      col0 + (c & 3) * 8) = v;
        }
        __syncwarp();
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

int attention_f16_tile_prepare_device() {
  return cuda_status(cudaFuncSetAttribute(attention_f16_tile_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemF));
}

int attention_f16_tile_launch(const CUtensorMap& tq, const CUtensorMap& tk,
                              const CUtensorMap& tvt, const AttnF16Args& a, cudaStream_t s) {
  const int grid = std::min(a.n_items, device_num_sms());
  if (int st = launch_kernel(attention_f16_tile_kernel, dim3(grid), dim3(kThreadsF), kSmemF, s, 1,
                             tq, tk, tvt, a))
    return st;
  return cuda_status(cudaGetLastError());
}

}  // namespace vitb200
