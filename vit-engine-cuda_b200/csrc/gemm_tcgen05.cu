// Split-operand GEMM on sm_100a tensor cores: Y = epilogue(A * B^T) with
// A = X[M][K], B = W[N][K] (PyTorch Linear layout), given either as TF32 hi/lo
// pairs (kind::tf32, three TF32 products per multiply) or as FP16 splits
// (kind::f16: A as hi, lo*2^11; W as hi, lo*2^11, hi*2^11 of W*s; three FP16
// products, all at the 2^11 scale, undone with an exact power of two in the
// epilogue). The TF32 description below holds for both kinds, with K slices of
// 16 and chunks of up to 256 for FP16.
//
// Reference math: the opt-in CuTe kernel csrc/kernels/gemm_cute_tf32.cu:104-125
// computes hi*hi + hi*lo + lo*hi per 32-wide K tile with mma.sync m16n8k8 and
// adds each tile's tensor-core result to an FP32 running sum in registers; the
// default path csrc/kernels/gemm.cu:12-96 is SIMT FP32 with the same epilogues
// (bias, erf-GELU). This kernel keeps that arithmetic — three TF32 products,
// lo*lo dropped, the tensor core accumulating only a short K chunk, chunks
// summed in round-to-nearest FP32 — and maps it onto Blackwell:
//
//  * persistent CTAs (one per SM), static round-robin over 128 x BN output tiles;
//  * warp 0: TMA producer. One 3-D bulk-tensor copy per operand per stage brings
//    the hi and lo planes of a [rows][BK] K-major tile (swizzled to the BK*4-byte
//    row) into a STAGES-deep shared-memory ring (mbarrier full/empty pairs);
//  * warp 1: allocates TMEM and, from one thread, issues tcgen05.mma.kind::tf32
//    (M=128, N=BN, K=8) — lo*hi, hi*lo, hi*hi per 8-wide K slice — into 512/BN
//    TMEM chunk accumulators used round robin; a chunk spans CHUNK_KB stages
//    (K = 128) and
//    starts from zero. The tensor core's accumulator truncates toward zero, so
//    keeping each chain short is what holds FP32-level accuracy;
//  * warps 4-7 and 8-11: two epilogue warpgroups, each owning half of the tile's
//    columns. Both drain every chunk (tcgen05.ld, one output row per thread)
//    into FP32 running sums in registers and free the TMEM buffer; after the
//    last chunk they apply bias / GELU / residual / positional add and store
//    fp32 and/or the TF32 pair the next GEMM consumes, while the MMA issuer
//    already fills the free chunk buffers with the next tile.
//
// Large problems run 256 x 256 tiles on CTA pairs (tcgen05 cta_group::2: the
// leader issues the MMAs, each CTA loads its own 128 rows of A and half of B).
// Small ones (fewer tiles than half the SMs) may split K over a thread-block
// cluster of d CTAs per tile: the others leave their partial tiles in their
// shared memory and the first adds them in split order over distributed
// shared memory. plan_gemm picks the tile configuration and the split.
//
// Every CTA loads its own tiles with plain per-CTA copies (no broadcast loads).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "engine.h"
#include "vitb200.h"

namespace vitb200 {

struct GemmArgs {
  int64_t M;
  int N;
  int Kp;
  int num_n_tiles;
  int num_tiles;
  int num_kb;
  int num_chunks;  // chunks per work unit
  int ksplit;      // K splits per output tile: a cluster of ksplit CTAs, one split each
  int kb_per;      // K blocks per work unit (num_kb / ksplit)
  int vec_out;     // fp32 output rows are 16-byte aligned (float4 stores)
  int vec_pair;    // pair rows are 16-byte aligned
  int vec_res;     // residual rows are 16-byte aligned
  int vec_h16;     // FP16-pair rows are 16-byte aligned
  int vec_bias;    // bias is 16-byte aligned
  float acc_scale; // F16 kernels: multiplies the accumulator (a power of two)
  int tma_h16;     // FP16 splits of the result go out through tmap_h (TMA stores):
                   // out_h16 (planes 0-1), or q16 | k16 (planes 0-1 | 2-3)
  int tma_out;     // the fp32 result goes out through tmap_h (TMA stores), and the
                   // residual (the same tensor) comes in through it (TMA loads)
  int tma_h16b;    // with tma_out: the FP16 split of the result through tmap_h2
  int* err;
  GemmEpilogue epi;
};

constexpr int kBM = 128;
// Folded LayerNorm: the most 32-column slabs a row's statistics come in
// (768 / 32; a multiple of 4).
constexpr int kMaxLnSlabs = 24;
// Epilogue transpose buffer of one warp: 32 rows x 32 words (pitch 32); the
// 16-byte chunk q of row r sits at chunk position q ^ (r & 7), so a lane
// writing its own row and eight lanes reading one row both touch eight
// different bank groups.
constexpr int kStgWords = 32 * 32;
__device__ __forceinline__ int stg_at(int r, int q) { return r * 32 + 4 * (q ^ (r & 7)); }
// Warpgroup 0 = TMA producer, MMA issuer, two idle warps; warpgroups 1..EPI =
// epilogue (EPI = 2, 3 or 4). Launched at kLaunchRegs registers per thread
// (65536 / threads, rounded down to 8), then warpgroup 0 gives registers up
// (kCtrlRegs) and the epilogue warpgroups take them (kEpiRegs):
//   EPI 2: 384 threads at 168: 128 * 56 + 256 * 224 = 64512 = 384 * 168
//   EPI 3: 512 threads at 128: 128 * 32 + 384 * 160 = 65536 = 512 * 128
//   EPI 4: 640 threads at  96: 128 * 56 + 512 * 104 = 60416 <= 640 * 96
// build.py checks that ptxas allocated exactly kLaunchRegs to each instance.
// The epilogue warpgroups take the tile's 32-column slabs round robin (slab s
// to warpgroup s % EPI). Every compiled configuration uses EPI = 2: four
// epilogue warpgroups, at 104 registers, spilled and ran 12-20 % slower, and
// three (CTA-pair tiles, 96 columns per thread at 160 registers) spilled too
// and ran 5-8 % slower on all four block GEMMs.
template <int EPI>
struct EpiCfg {
  static constexpr int kThreads = 128 * (1 + EPI);
  static constexpr uint32_t kLaunchRegs = EPI == 2 ? 168 : (EPI == 3 ? 128 : 96);
  static constexpr uint32_t kCtrlRegs = EPI == 3 ? 32 : 56;
  static constexpr uint32_t kEpiRegs = EPI == 2 ? 224 : (EPI == 3 ? 160 : 104);
  static_assert(EPI >= 2 && EPI <= 4, "epilogue warpgroups");
  static_assert(128 * kCtrlRegs + 128 * EPI * kEpiRegs <= kThreads * kLaunchRegs,
                "register split exceeds the launch allocation");
  static_assert(kThreads * kLaunchRegs <= 65536, "registers");
};
constexpr int kTmemAll = 512;  // TMEM columns: chunk accumulators of BN columns each

// Operand kinds: TF32 pairs; FP16 splits with B's third plane hi*2^11 (one
// accumulator takes all three products); FP16 splits with two B planes, the
// cross products accumulated first and folded in by scale-input-d (every
// stage is one chunk).
enum OperandKind : int { kKindTF32 = 0, kKindF16 = 1, kKindF16SD = 2 };

template <int KIND, int BN, int BK, int STAGES, int CHUNK_KB, bool PAIR, int EPI = 2>
struct GemmCfg {
  static constexpr bool F16 = KIND != kKindTF32;
  static constexpr bool SD = KIND == kKindF16SD;
  // PAIR: the two CTAs of a cluster share a 256 x BN tile; each holds 128 rows
  // of A, BN/2 rows of B and 128 x BN accumulators in its own TMEM.
  // F16: operands are FP16 splits (A: hi, lo; B: hi, lo, hi*2^11), TF32
  // otherwise (A and B: hi, lo).
  static constexpr int kEs = F16 ? 2 : 4;       // bytes per element
  static constexpr int kRowBytes = BK * kEs;    // one K-major tile row
  static constexpr int kMmaK = F16 ? 16 : 8;    // K per tcgen05.mma (32 bytes)
  static constexpr int kBPlanes = KIND == kKindF16 ? 3 : 2;
  static constexpr int kBRows = PAIR ? BN / 2 : BN;
  static constexpr int kAPlane = kBM * BK * kEs;  // bytes of one A plane
  static constexpr int kBPlane = kBRows * BK * kEs;
  static constexpr int kStageBytes = 2 * kAPlane + kBPlanes * kBPlane;
  // Per epilogue warp: a 32 x 32 transpose buffer (row pitch 36 floats keeps the
  // 16-byte row writes and the transposed reads free of bank conflicts).
  static constexpr int kStagingBytes = 4 * EPI * kStgWords * 4;
  static constexpr int kSmemBytes = STAGES * kStageBytes + kStagingBytes + 1024;
  static constexpr int kNumBufs = kTmemAll / BN;  // chunk accumulators in TMEM
  static constexpr int kTmemCols = kTmemAll;
  static constexpr int kSlabs = BN / 32;          // 32-column slabs of a tile
  static constexpr int kWgSlabs = (kSlabs + EPI - 1) / EPI;  // slabs per epilogue warpgroup (max)
  static constexpr int kWgCols = 32 * kWgSlabs;   // FP32 sums per epilogue thread
  static constexpr int kTileM = PAIR ? 2 * kBM : kBM;
  static constexpr uint32_t kIdesc = F16 ? make_idesc_f16(kTileM, BN) : make_idesc_tf32(kTileM, BN);
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert(!PAIR || BN % 16 == 0, "pair N");
  static_assert(kRowBytes == 128 || kRowBytes == 64, "BK row must be a 64B or 128B swizzle span");
  static_assert((kTmemCols & (kTmemCols - 1)) == 0 && kTmemCols >= 32 && kTmemCols <= 512,
                "TMEM columns must be a power of two in [32, 512]");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
  // split-K partial sums of a CTA (128 x BN fp32) fit in its stage ring
  static_assert(128 * BN * 4 <= STAGES * kStageBytes, "split-K partials");
  static_assert(CHUNK_KB >= 1, "chunk");
  static_assert(!SD || CHUNK_KB == 1, "scale-input-d needs one stage per chunk");
};

// Epilogue of one 32 x 32 slab, warp-collective: lane i holds row m_base + i,
// columns n0..n0+31, in v (accumulator in, final values out):
// bias -> GELU -> (positional row | column split) -> residual -> fp32 / TF32-pair
// stores. The order of additions follows the reference: residual + (acc + bias)
// (vit_cuda/model.py:48,60) and (conv + bias) + pos (pos_encoding.cu:20-26).
// Row-contiguous outputs go through the warp's transpose buffer `stg`, so every
// global access instruction covers four whole 128-byte row segments instead of
// sixteen bytes of 32 different rows.
// Stores the FP16 split of a warp's 32 x 32 slab (lane i = row m_base + i,
// values v) as planes base[p * plane + row * ld + col_base ..]: hi and
// lo * 2^11. Through the warp's transpose buffer: chunks 0-3 of a row hold hi
// halves, 4-7 lo halves; lanes 0-3 of each group of eight store a row's hi
// (64 B), lanes 4-7 its lo, four rows per instruction.
__device__ __forceinline__ void h16_slab_store(const float (&v)[32], float* stg, int lane,
                                               int64_t m_base, int64_t M, uint16_t* base,
                                               int64_t ld, int64_t plane, int64_t col_base) {
  const int rsub = lane >> 3;
  const int q = lane & 7;  // this lane's 16-byte chunk of a row when flushing
#pragma unroll
  for (int j = 0; j < 32; j += 8) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) h16_split2(v[j + 2 * t], v[j + 2 * t + 1], hw[t], lw[t]);
    *reinterpret_cast<uint4*>(stg + stg_at(lane, j / 8)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(stg + stg_at(lane, 4 + j / 8)) =
        make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
  __syncwarp();
  const int pl = q >> 2;         // 0: hi, 1: lo
  const int hcol = (q & 3) * 8;  // first of this lane's eight columns
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int r = 4 * k + rsub;
    const int64_t mr = m_base + r;
    const uint4 t = *reinterpret_cast<const uint4*>(stg + stg_at(r, q));
    if (mr < M) *reinterpret_cast<uint4*>(base + pl * plane + mr * ld + col_base + hcol) = t;
  }
  __syncwarp();
}

// The same split through a TMA tensor store: the warp writes its slab into
// its 4 KB transpose buffer in the layout of the map's box {32 columns, 32
// rows, 2 planes} with the 64-byte swizzle (16-byte chunk q of row r at
// chunk q ^ ((r >> 1) & 3): conflict-free), and lane 0 stores it. Before the
// buffer is written again lane 0 waits until the previous store has read it;
// rows past M are clipped by the map.
__device__ __forceinline__ void h16_slab_store_tma(const float (&v)[32], float* stg, int lane,
                                                   int64_t m_base, int64_t col_base,
                                                   const CUtensorMap* tmap_h, int plane0) {
  uint8_t* buf = reinterpret_cast<uint8_t*>(stg);
  if (lane == 0) bulk_wait_group_read<0>();
  __syncwarp();
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) h16_split2(v[8 * q + 2 * t], v[8 * q + 2 * t + 1], hw[t], lw[t]);
    const int at = lane * 64 + 16 * (q ^ sw);
    *reinterpret_cast<uint4*>(buf + at) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(buf + 2048 + at) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_3d(tmap_h, buf, static_cast<int>(col_base), static_cast<int>(m_base), plane0);
    bulk_commit_group();
  }
}

__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* err);

// Row statistics (count 32, sum, M2 about the mean) of one lane's 32 values,
// four independent chains each.
__device__ __forceinline__ float2 slab_stats(const float (&v)[32]) {
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 32; ++j) s4[j & 3] += v[j];
  const float sum = (s4[0] + s4[1]) + (s4[2] + s4[3]);
  const float mean = sum * (1.f / 32.f);
  float q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float d = v[j] - mean;
    q4[j & 3] = fmaf(d, d, q4[j & 3]);
  }
  return make_float2(sum, (q4[0] + q4[1]) + (q4[2] + q4[3]));
}

template <bool F16>
__device__ __forceinline__ void epilogue_slab(const GemmArgs& a, int64_t m_base, int lane, int n0,
                                              float (&v)[32], float* stg,
                                              const CUtensorMap* tmap_h,
                                              const CUtensorMap* tmap_h2, uint64_t* res_bar,
                                              uint32_t& res_phase, float ln_mu, float ln_rstd) {
  const GemmEpilogue& e = a.epi;
  const int N = a.N;
  const int64_t m = m_base + lane;
  const bool row_ok = m < a.M;
  const bool full = (n0 + 32 <= N);

  // Undo the operand scales (FP16 kinds; a power of two, so the product is
  // exact) and add the bias: one rounding, as acc * scale + bias would give.
  const float sc = F16 ? a.acc_scale : 1.f;
  if (e.ln_c != nullptr) {
    // LayerNorm folded in: rstd * (acc - mean * c) + d.
    if (full) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 c4 = __ldg(reinterpret_cast<const float4*>(e.ln_c + n0 + j));
        const float4 d4 = __ldg(reinterpret_cast<const float4*>(e.ln_d + n0 + j));
        v[j] = fmaf(ln_rstd, fmaf(-ln_mu, c4.x, v[j] * sc), d4.x);
        v[j + 1] = fmaf(ln_rstd, fmaf(-ln_mu, c4.y, v[j + 1] * sc), d4.y);
        v[j + 2] = fmaf(ln_rstd, fmaf(-ln_mu, c4.z, v[j + 2] * sc), d4.z);
        v[j + 3] = fmaf(ln_rstd, fmaf(-ln_mu, c4.w, v[j + 3] * sc), d4.w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = n0 + j;
        const float c = n < N ? __ldg(e.ln_c + n) : 0.f;
        const float d = n < N ? __ldg(e.ln_d + n) : 0.f;
        v[j] = fmaf(ln_rstd, fmaf(-ln_mu, c, v[j] * sc), d);
      }
    }
  } else if (e.bias != nullptr) {
    if (full && a.vec_bias) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 b4 = __ldg(reinterpret_cast<const float4*>(e.bias + n0 + j));
        v[j] = fmaf(v[j], sc, b4.x);
        v[j + 1] = fmaf(v[j + 1], sc, b4.y);
        v[j + 2] = fmaf(v[j + 2], sc, b4.z);
        v[j + 3] = fmaf(v[j + 3], sc, b4.w);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = n0 + j;
        v[j] = fmaf(v[j], sc, (n < N) ? __ldg(e.bias + n) : 0.f);
      }
    }
  } else if constexpr (F16) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = v[j] * sc;
  }
  if (e.gelu) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
  }

  if (e.mode == kModeQKVAttn16) {
    // q | k | v column thirds (E % 64 == 0: slabs are full and never straddle).
    const int E = e.e_split;
    const int part = n0 / E;
    const float sc = part == 0 ? e.q_scale : (part == 1 ? e.k_scale : e.v_scale);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = v[j] * sc;  // exact: a power of two
    if (part < 2) {
      if (a.tma_h16)  // q and k: planes 0-1 and 2-3 of one map
        h16_slab_store_tma(v, stg, lane, m_base, n0 - part * E, tmap_h, 2 * part);
      else
        h16_slab_store(v, stg, lane, m_base, a.M, part == 0 ? e.q16 : e.k16, E, a.M * E,
                       n0 - part * E);
      return;
    }
    // V: transposed per (image, head); lanes hold consecutive tokens, so each
    // column's store is one contiguous 64-byte run per plane.
    if (!row_ok) return;
    const int vc = n0 - 2 * E;
    const int64_t bimg = m / e.T;
    const int64_t t = m - bimg * e.T;
    const int64_t head_row = (bimg * (E / 64) + vc / 64) * 64 + (vc & 63);
    __half* dst = reinterpret_cast<__half*>(e.vt16) + head_row * e.T4 + t;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      __half hi, lo;
      h16_split(v[j], hi, lo);
      const int64_t o = static_cast<int64_t>(j) * e.T4;
      dst[o] = hi;
      dst[o + e.vt16_plane] = lo;
    }
    return;
  }

  if (e.mode == kModeQKVAttn && n0 >= 2 * e.e_split) {
    // V columns: TF32 pair of V transposed per (image, head). Lanes hold
    // consecutive rows, so each column's store is one coalesced line.
    if (!row_ok) return;
    const int vc = n0 - 2 * e.e_split;
    const int64_t bimg = m / e.T;
    const int64_t t = m - bimg * e.T;
    const int64_t head_row = (bimg * (e.e_split / 64) + vc / 64) * 64 + (vc & 63);
    float* dst = e.vt_pair + head_row * e.T4 + t;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      float hi, lo;
      tf32_split(v[j], hi, lo);
      dst[static_cast<int64_t>(j) * e.T4] = hi;
      dst[static_cast<int64_t>(j) * e.T4 + e.vt_plane] = lo;
    }
    return;
  }

  int64_t plane_off = 0;
  int64_t col_base = n0;
  if (e.mode == kModeSplit3) {
    const int plane = n0 / e.e_split;  // e_split % 32 == 0: a slab never straddles
    plane_off = static_cast<int64_t>(plane) * e.split_plane;
    col_base = n0 - plane * e.e_split;
  }

  const bool staged = full && e.mode != kModePatch && (!e.out || a.vec_out) &&
                      (!e.out_pair || a.vec_pair) && (!e.residual || a.vec_res) &&
                      (!e.out_h16 || a.vec_h16);
  if (staged) {
    const int rsub = lane >> 3;        // row within a group of four
    const int q = lane & 7;            // this lane's 16-byte chunk of a 32-column row
    const int c4 = q * 4;
    // TMA path: the buffer's layout (chunk q of row r at q ^ (r & 7)) is the
    // map's 128-byte swizzle of the box {32 columns, 32 rows}. Before it is
    // written again, the previous slab's store must have read it.
    if (a.tma_out) {
      if (lane == 0) bulk_wait_group_read<0>();
      __syncwarp();
    }
    if (e.residual != nullptr) {
      if (a.tma_out) {
        // The residual slab (rows past M read as zeros) in one load.
        if (lane == 0) {
          mbar_arrive_expect_tx(res_bar, 32 * 32 * 4);
          tma_load_3d(stg, tmap_h, res_bar, static_cast<int>(col_base), static_cast<int>(m_base),
                      0);
        }
        // Every lane waits (acquire) before reading the slab; a wait that
        // gives up records its code and lets the copy land before going on.
        if (!mbar_wait(res_bar, res_phase, a.err, kErrWaitFull))
          drain_wait(res_bar, res_phase, a.err);
        res_phase ^= 1u;
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int r = 4 * k + rsub;
          const int64_t mr = m_base + r;
          float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
          if (mr < a.M)
            t = *reinterpret_cast<const float4*>(e.residual + mr * e.ldr + col_base + c4);
          *reinterpret_cast<float4*>(stg + stg_at(r, q)) = t;
        }
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 t = *reinterpret_cast<const float4*>(stg + stg_at(lane, j / 4));
        v[j] = t.x + v[j];
        v[j + 1] = t.y + v[j + 1];
        v[j + 2] = t.z + v[j + 2];
        v[j + 3] = t.w + v[j + 3];
      }
      __syncwarp();
    }
    // Writes the warp's 32 rows from the buffer: 8 instructions, 4 rows each.
    auto flush = [&](float* base, int64_t ld) {
      __syncwarp();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int r = 4 * k + rsub;
        const int64_t mr = m_base + r;
        const float4 t = *reinterpret_cast<const float4*>(stg + stg_at(r, q));
        if (mr < a.M) *reinterpret_cast<float4*>(base + mr * ld + col_base + c4) = t;
      }
      __syncwarp();
    };
    if (e.out != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(stg + stg_at(lane, j / 4)) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      if (a.tma_out) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(tmap_h, stg, static_cast<int>(col_base), static_cast<int>(m_base), 0);
          bulk_commit_group();
        }
      } else {
        flush(e.out + plane_off, e.ldo);
      }
    }
    if (e.out_pair != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(stg + stg_at(lane, j / 4)) =
            make_float4(tf32_round(v[j]), tf32_round(v[j + 1]), tf32_round(v[j + 2]),
                        tf32_round(v[j + 3]));
      flush(e.out_pair, e.ldp);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 l;
        float h;
        tf32_split(v[j], h, l.x);
        tf32_split(v[j + 1], h, l.y);
        tf32_split(v[j + 2], h, l.z);
        tf32_split(v[j + 3], h, l.w);
        *reinterpret_cast<float4*>(stg + stg_at(lane, j / 4)) = l;
      }
      flush(e.out_pair + e.pair_plane, e.ldp);
    }
    if (e.stats_out != nullptr) {
      const float2 st = slab_stats(v);
      if (m < a.M) e.stats_out[static_cast<int64_t>(n0 / 32) * a.M + m] = st;
      if (e.h16_check) {
        // fmaxf drops NaN; the slab's sum carries it.
        float mx = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) mx = fmaxf(mx, fabsf(v[j]));
        if (row_ok && !(mx < kH16Limit && st.x == st.x)) report_error(a.err, kErrF16Range);
      }
    }
    if (e.out_h16 != nullptr) {
      if (a.tma_out) {  // the fp32 store must have read the buffer
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
      }
      if (a.tma_h16)
        h16_slab_store_tma(v, stg, lane, m_base, col_base, tmap_h, 0);
      else if (a.tma_h16b)
        h16_slab_store_tma(v, stg, lane, m_base, col_base, tmap_h2, 0);
      else
        h16_slab_store(v, stg, lane, m_base, a.M, e.out_h16, e.ldh, e.h16_plane, col_base);
    }
    return;
  }

  if (e.mode == kModePatch && full && e.out && a.vec_out && !e.out_pair && !e.out_h16 &&
      !e.residual && N % 4 == 0 && reinterpret_cast<uintptr_t>(e.pos) % 16 == 0) {
    // Patch rows through the transpose buffer: each row's positional row is
    // added, and row m = b * P + p is stored as token row b * T + 1 + p.
    const int rsub = lane >> 3;
    const int q = lane & 7;
    const int c4 = q * 4;
    // (image, patch) of this lane's rows m_base + rsub + 4k, stepped without
    // a division per row.
    const int64_t m0 = m_base + rsub;
    const int64_t b0 = m0 / e.P;
    const int p0 = static_cast<int>(m0 - b0 * e.P);
    int64_t bk = b0;
    int pk = p0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = 4 * k + rsub;
      const int64_t mr = m_base + r;
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (mr < a.M)
        t = *reinterpret_cast<const float4*>(e.pos + static_cast<int64_t>(1 + pk) * N +
                                              col_base + c4);
      *reinterpret_cast<float4*>(stg + stg_at(r, q)) = t;
      pk += 4;
      while (pk >= e.P) {
        pk -= e.P;
        ++bk;
      }
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const float4 t = *reinterpret_cast<const float4*>(stg + stg_at(lane, j / 4));
      *reinterpret_cast<float4*>(stg + stg_at(lane, j / 4)) =
          make_float4(v[j] + t.x, v[j + 1] + t.y, v[j + 2] + t.z, v[j + 3] + t.w);
    }
    __syncwarp();
    bk = b0;
    pk = p0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = 4 * k + rsub;
      const int64_t mr = m_base + r;
      const float4 t = *reinterpret_cast<const float4*>(stg + stg_at(r, q));
      if (mr < a.M) {
        const int64_t orow = bk * e.T + 1 + pk;
        *reinterpret_cast<float4*>(e.out + orow * e.ldo + col_base + c4) = t;
      }
      pk += 4;
      while (pk >= e.P) {
        pk -= e.P;
        ++bk;
      }
    }
    __syncwarp();
    return;
  }

  // Generic path (partial slab, positional rows, unaligned outputs): per row.
  if (!row_ok) return;
  int64_t out_row = m;
  if (e.mode == kModePatch) {
    const int64_t b = m / e.P;
    const int p = static_cast<int>(m - b * e.P);
    out_row = b * e.T + 1 + p;
    const float* pos_row = e.pos + static_cast<int64_t>(1 + p) * N;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = n0 + j;
      v[j] = v[j] + ((n < N) ? __ldg(pos_row + n) : 0.f);
    }
  }
  if (e.residual != nullptr) {
    const float* r = e.residual + out_row * e.ldr + col_base;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < N) v[j] = r[j] + v[j];
  }
  if (e.out != nullptr) {
    float* o = e.out + plane_off + out_row * e.ldo + col_base;
    if (full && a.vec_out) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < N) o[j] = v[j];
    }
  }
  if (e.out_pair != nullptr) {
    float* ph = e.out_pair + out_row * e.ldp + col_base;
    float* pl = ph + e.pair_plane;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < N) {
        float h, l;
        tf32_split(v[j], h, l);
        ph[j] = h;
        pl[j] = l;
      }
  }
  if (e.out_h16 != nullptr) {
    __half* ph = reinterpret_cast<__half*>(e.out_h16) + out_row * e.ldh + col_base;
    __half* pl = ph + e.h16_plane;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n0 + j < N) h16_split(v[j], ph[j], pl[j]);
  }
}

// TMEM chunk buffer of chunk j of this CTA's local tile `local`: chunks use
// the kNumBufs buffers round robin. Both epilogue warpgroups drain every chunk
// (each its half of the columns) and the MMA issuer refills buffers in order,
// so every barrier is waited on phase after phase by each of its waiters.
template <int NBUF>
__device__ __forceinline__ void chunk_slot(int local, int j, int num_chunks, int& buf,
                                           uint32_t& use) {
  const uint32_t seq = static_cast<uint32_t>(local * num_chunks + j);
  buf = static_cast<int>(seq % NBUF);
  use = seq / NBUF;
}

// Lane 0 waits; the verdict is broadcast so the warp stays converged for the
// .sync.aligned tcgen05 instructions that follow.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                          int lane) {
  int ok = 1;
  if (lane == 0) ok = mbar_wait(bar, parity, err, code) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
}

// Time-bounded wait used on the way out; it ignores the error word because
// its purpose is to let in-flight asynchronous work land before the CTA exits.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t addr = smem_addr(bar);
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(addr, parity)) {
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      report_error(err, kErrDrain);
      return;
    }
  }
}

template <int KIND, int BN, int BK, int STAGES, int CHUNK_KB, bool PAIR, int EPI>
__global__ void __launch_bounds__(EpiCfg<EPI>::kThreads, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_b,
                       const __grid_constant__ CUtensorMap tmap_h,
                       const __grid_constant__ CUtensorMap tmap_h2, const GemmArgs args) {
  using Cfg = GemmCfg<KIND, BN, BK, STAGES, CHUNK_KB, PAIR, EPI>;
  using Epi = EpiCfg<EPI>;
  constexpr bool F16 = Cfg::F16;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t chunk_full_bar[Cfg::kNumBufs];
  __shared__ __align__(8) uint64_t chunk_empty_bar[Cfg::kNumBufs];
  __shared__ __align__(8) uint64_t mma_done_bar;
  __shared__ __align__(8) uint64_t split_bar[4 * EPI];  // split-K: other CTAs' partials ready
  __shared__ __align__(8) uint64_t res_bar[4 * EPI];    // per epilogue warp: residual slab landed
  __shared__ uint32_t tmem_base_slot;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = args.err;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // rank 0 issues the pair's MMAs
  const bool leader = rank == 0;
  // Work units: a CTA (single) or a cluster of two (pair) per output tile.
  const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int num_units = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  // 1024-byte aligned ring base (swizzle atoms are 8 rows x 128 B).
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* ring = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < Cfg::kNumBufs; ++b) {
      mbar_init(&chunk_full_bar[b], 1);
      // one arrival per draining warp (4 * EPI per CTA, of both CTAs for a pair)
      mbar_init(&chunk_empty_bar[b], (PAIR ? 2 : 1) * 4 * EPI);
    }
    mbar_init(&mma_done_bar, 1);
    for (int i = 0; i < 4 * EPI; ++i) mbar_init(&res_bar[i], 1);
    if (!PAIR && args.ksplit > 1) {
      // one arrival per lane of each other CTA's slab warp
      for (int i = 0; i < 4 * EPI; ++i) mbar_init(&split_bar[i], 32 * (args.ksplit - 1));
    }
    fence_barrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  // Peer barriers initialised before any remote use (CTA pair, split-K cluster).
  if (PAIR || args.ksplit > 1) cluster_sync_all();
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(&tmem_base_slot, Cfg::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(&tmem_base_slot, Cfg::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_slot;
  griddep_wait();
  griddep_launch_dependents();

  const int num_tiles = args.num_tiles;
  const int num_chunks = args.num_chunks;
  // Work unit w: output tile w / ksplit, K blocks [(w % ksplit) * kb_per, +kb_per).
  const int ksplit = args.ksplit;
  const int kb_per = args.kb_per;
  const int num_work = num_tiles * ksplit;

  if (warp < 4) {
  // Control warpgroup: gives registers to the epilogue warpgroups.
  setmaxnreg_dec<Epi::kCtrlRegs>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int w = unit; w < num_work && ok; w += num_units) {
        const int tile = w / ksplit;
        const int kb0 = (w - tile * ksplit) * kb_per;
        const int m_blk = tile / args.num_n_tiles;
        const int n_blk = tile - m_blk * args.num_n_tiles;
        const int a_row = m_blk * Cfg::kTileM + static_cast<int>(rank) * kBM;
        const int b_row = n_blk * BN + static_cast<int>(rank) * Cfg::kBRows;
        for (int kb = kb0; kb < kb0 + kb_per; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = ring + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + 2 * Cfg::kAPlane;
          if constexpr (PAIR) {
            // Both CTAs' copies complete on the leader's barrier, which expects
            // the bytes of both.
            const uint32_t full_leader = mapa_shared(smem_addr(&full_bar[stage]), 0);
            if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * Cfg::kStageBytes);
            tma_load_3d_pair(sa, &tmap_a, full_leader, kb * BK, a_row, 0);
            tma_load_3d_pair(sb, &tmap_b, full_leader, kb * BK, b_row, 0);
          } else {
            mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageBytes);
            tma_load_3d(sa, &tmap_a, &full_bar[stage], kb * BK, a_row, 0);
            tma_load_3d(sb, &tmap_b, &full_bar[stage], kb * BK, b_row, 0);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Let every copy issued land before the CTAs can exit (the leader's
      // barriers count the bytes of both CTAs of a pair).
      if (leader) {
        for (int s = 0; s < STAGES; ++s) {
          if (issued > s) {
            const int64_t fills = (issued - s + STAGES - 1) / STAGES;
            drain_wait(&full_bar[s], static_cast<uint32_t>((fills - 1) & 1), err);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      // Arrive on a barrier of this CTA and, for a pair, on the same barrier of
      // the peer, once the MMAs issued so far complete.
      auto commit = [&](uint64_t* bar) {
        if constexpr (PAIR) {
          const uint32_t a = smem_addr(bar);
          umma_commit_pair(a);
          umma_commit_pair(mapa_shared(a, 1));
        } else {
          umma_commit(bar);
        }
      };
      for (int w = unit; w < num_work && ok; w += num_units, ++local) {
        for (int kb = 0; kb < kb_per; ++kb) {  // relative to the work unit's first K block
          const int j = kb / CHUNK_KB;
          const bool chunk_first = (kb - j * CHUNK_KB) == 0;
          const bool chunk_last = (kb - j * CHUNK_KB) == CHUNK_KB - 1 || kb == kb_per - 1;
          int buf;
          uint32_t use;
          chunk_slot<Cfg::kNumBufs>(local, j, num_chunks, buf, use);
          if (chunk_first) {
            if (!mbar_wait(&chunk_empty_bar[buf], (use & 1u) ^ 1u, err, kErrWaitAccEmpty)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          if (!mbar_wait(&full_bar[stage], phase, err, kErrWaitFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
          const uint32_t a_hi = smem_addr(ring + stage * Cfg::kStageBytes);
          const uint32_t a_lo = a_hi + Cfg::kAPlane;
          const uint32_t b_hi = a_hi + 2 * Cfg::kAPlane;
          const uint32_t b_lo = b_hi + Cfg::kBPlane;
          // hi * hi: TF32 and scale-input-d use B's hi plane; F16 its third
          // plane, hi * 2^11.
          const uint32_t b_hh = KIND == kKindF16 ? b_hi + 2 * Cfg::kBPlane : b_hi;
          auto mma = [&](uint64_t da, uint64_t db, uint32_t acc) {
            if constexpr (F16 && PAIR) {
              umma_f16_pair(d_tmem, da, db, Cfg::kIdesc, acc);
            } else if constexpr (F16) {
              umma_f16(d_tmem, da, db, Cfg::kIdesc, acc);
            } else if constexpr (PAIR) {
              umma_tf32_pair(d_tmem, da, db, Cfg::kIdesc, acc);
            } else {
              umma_tf32(d_tmem, da, db, Cfg::kIdesc, acc);
            }
          };
          // Descriptors of the stage's first K slice; one MMA's K further is
          // +32 bytes, i.e. +2 in the descriptor's address field.
          const uint64_t dah = make_sdesc_kmajor(a_hi, Cfg::kRowBytes);
          const uint64_t dal = make_sdesc_kmajor(a_lo, Cfg::kRowBytes);
          const uint64_t dbh = make_sdesc_kmajor(b_hi, Cfg::kRowBytes);
          const uint64_t dbl = make_sdesc_kmajor(b_lo, Cfg::kRowBytes);
          const uint64_t dbhh = make_sdesc_kmajor(b_hh, Cfg::kRowBytes);
          if constexpr (Cfg::SD) {
            // The stage's cross products (each scaled by 2^11) first, then
            // hi * hi with the accumulator scaled by 2^-11 on the first one.
#pragma unroll
            for (int kk = 0; kk < BK / Cfg::kMmaK; ++kk) {
              const uint64_t o = static_cast<uint64_t>(2 * kk);
              mma(dal + o, dbh + o, kk == 0 ? 0u : 1u);  // lo * hi
              mma(dah + o, dbl + o, 1u);                 // hi * lo
            }
#pragma unroll
            for (int kk = 0; kk < BK / Cfg::kMmaK; ++kk) {
              const uint64_t o = static_cast<uint64_t>(2 * kk);
              if (kk == 0) {
                if constexpr (PAIR) {
                  umma_f16_pair_sd11(d_tmem, dah, dbh, Cfg::kIdesc);
                } else {
                  umma_f16_sd11(d_tmem, dah, dbh, Cfg::kIdesc);
                }
              } else {
                mma(dah + o, dbh + o, 1u);  // hi * hi
              }
            }
          } else {
#pragma unroll
            for (int kk = 0; kk < BK / Cfg::kMmaK; ++kk) {
              const uint64_t o = static_cast<uint64_t>(2 * kk);
              const uint32_t acc0 = (chunk_first && kk == 0) ? 0u : 1u;
              mma(dal + o, dbh + o, acc0);  // lo * hi
              mma(dah + o, dbl + o, 1u);    // hi * lo
              mma(dah + o, dbhh + o, 1u);   // hi * hi
            }
          }
          commit(&empty_bar[stage]);  // frees the stage once these MMAs finish
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (chunk_last) commit(&chunk_full_bar[buf]);
        }
      }
      // Every MMA this thread issued must finish before TMEM is released.
      if constexpr (PAIR) {
        umma_commit_pair(smem_addr(&mma_done_bar));
      } else {
        umma_commit(&mma_done_bar);
      }
      drain_wait(&mma_done_bar, 0, err);
    }
  }
  } else {
    setmaxnreg_inc<Epi::kEpiRegs>();
    // ------------------------------------------------------------ epilogue
    // Warps 4 .. 4 + 4*EPI - 1: warp w reads TMEM lanes [32*(w%4), +32) (one
    // output row per thread); epilogue warpgroup `wg` owns the tile's slabs
    // wg, wg + EPI, wg + 2*EPI, ... (32 columns each).
    const int wg = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    float* stg = reinterpret_cast<float*>(ring + STAGES * Cfg::kStageBytes) +
                 (warp - 4) * kStgWords;
    uint32_t res_phase = 0;  // parity of this warp's next residual load (TMA path)
    int local = 0;
    bool ok = true;
    for (int w = unit; w < num_work && ok; w += num_units, ++local) {
      const int tile = w / ksplit;
      const int split = w - tile * ksplit;
      const int m_blk = tile / args.num_n_tiles;
      const int n_blk = tile - m_blk * args.num_n_tiles;
      // Folded LayerNorm: this row's mean and 1 / sqrt(var + eps), combined
      // from its slabs' (sum, M2) as Chan et al.'s parallel variance (every
      // slab holds 32 values: M2 = sum_s M2_s + 32 (m_s - mean)^2). Computed
      // before the accumulator is drained, so the loads overlap the MMAs; all
      // of a row's slabs (up to kMaxLnSlabs) are loaded at once.
      float ln_mu = 0.f, ln_rstd = 0.f;
      if (args.epi.ln_c != nullptr) {
        const int64_t m_row = static_cast<int64_t>(m_blk) * Cfg::kTileM +
                              static_cast<int64_t>(rank) * kBM + quarter * 32 + lane;
        if (m_row < args.M) {
          const float2* st = args.epi.ln_stats + m_row;
          const int slabs = args.epi.ln_slabs;
          float2 pr[kMaxLnSlabs];
#pragma unroll
          for (int sl = 0; sl < kMaxLnSlabs; ++sl)
            pr[sl] = sl < slabs ? st[static_cast<int64_t>(sl) * args.M] : make_float2(0.f, 0.f);
          float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
#pragma unroll
          for (int sl = 0; sl < kMaxLnSlabs; sl += 4) {
            t0 += pr[sl].x;
            t1 += pr[sl + 1].x;
            t2 += pr[sl + 2].x;
            t3 += pr[sl + 3].x;
          }
          const float n = 32.f * static_cast<float>(slabs);
          const float mean = ((t0 + t1) + (t2 + t3)) / n;
          float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
          auto acc = [&](float& q, float2 p2, bool valid) {
            const float d = fmaf(p2.x, 1.f / 32.f, -mean);
            if (valid) q += fmaf(32.f * d, d, p2.y);
          };
#pragma unroll
          for (int sl = 0; sl < kMaxLnSlabs; sl += 4) {
            acc(q0, pr[sl], sl < slabs);
            acc(q1, pr[sl + 1], sl + 1 < slabs);
            acc(q2, pr[sl + 2], sl + 2 < slabs);
            acc(q3, pr[sl + 3], sl + 3 < slabs);
          }
          const float var = ((q0 + q1) + (q2 + q3)) / n;
          ln_mu = mean;
          ln_rstd = 1.0f / sqrtf(var + args.epi.ln_eps);
        }
      }
      float sum[Cfg::kWgCols];
#pragma unroll
      for (int c = 0; c < Cfg::kWgCols; ++c) sum[c] = 0.f;
      for (int j = 0; j < num_chunks; ++j) {
        int buf;
        uint32_t use;
        chunk_slot<Cfg::kNumBufs>(local, j, num_chunks, buf, use);
        if (!warp_wait(&chunk_full_bar[buf], use & 1u, err, kErrWaitAccFull, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int i = 0; i < Cfg::kWgSlabs; ++i) {
          const int slab = wg + EPI * i;
          if (Cfg::kSlabs % EPI == 0 || slab < Cfg::kSlabs) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float part[16];
              __syncwarp();
              tmem_ld_32x32b_x16(
                  lane_base + static_cast<uint32_t>(buf * BN + slab * 32 + h * 16), part);
#pragma unroll
              for (int c = 0; c < 16; ++c) sum[i * 32 + h * 16 + c] += part[c];
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (PAIR && !leader) {
            mbar_arrive_cluster(mapa_shared(smem_addr(&chunk_empty_bar[buf]), 0));
          } else {
            mbar_arrive(&chunk_empty_bar[buf]);
          }
        }
      }
      if (!ok) break;
      if constexpr (!PAIR) {
        if (ksplit > 1) {
          // Split K over a cluster of ksplit CTAs, one work unit each (split =
          // cluster rank). Each warp slab (this warp's 32 rows x kWgCols
          // columns) is finished by one CTA of the cluster, `owner`, so that
          // the reduction and the epilogue are shared out: the other CTAs leave
          // their partial sums of it in their own stage ring, idle now that
          // their last MMA has completed, and the owner adds all partials in
          // split order over distributed shared memory (deterministic, the
          // same order whichever CTA adds). Layout [warp][c / 4][lane] of
          // float4: each warp access is 512 contiguous bytes.
          const int slab = warp - 4;
          const int owner = slab % ksplit;
          float4* part = reinterpret_cast<float4*>(ring) + slab * (Cfg::kWgCols / 4) * 32 + lane;
          // Split 0 keeps its partial in registers when it owns the slab;
          // every other partial is published (an owner other than split 0
          // reads its own back in its place in the order).
          if (split != 0 || owner != 0) {
            fence_proxy_async_smem();
#pragma unroll
            for (int c = 0; c < Cfg::kWgCols; c += 4)
              part[(c / 4) * 32] = make_float4(sum[c], sum[c + 1], sum[c + 2], sum[c + 3]);
          }
          if (split != owner) {
            mbar_arrive_cluster(
                mapa_shared(smem_addr(&split_bar[slab]), static_cast<uint32_t>(owner)));
            continue;
          }
          const bool got = mbar_wait_acq_cluster(&split_bar[slab], 0, err, kErrWaitSplit);
          if (!__all_sync(0xffffffffu, got)) {
            ok = false;
            break;
          }
          // sum = p_0 + p_1 + ... in split order.
          const uint32_t part_addr = smem_addr(part);
          if (split != 0) {
            const uint32_t src = mapa_shared(part_addr, 0u);
#pragma unroll
            for (int c = 0; c < Cfg::kWgCols; c += 4) {
              const float4 t = ld_shared_cluster_f4(src + static_cast<uint32_t>(c / 4) * 512u);
              sum[c] = t.x;
              sum[c + 1] = t.y;
              sum[c + 2] = t.z;
              sum[c + 3] = t.w;
            }
          }
          for (int sp = 1; sp < ksplit; ++sp) {
            const uint32_t src = mapa_shared(part_addr, static_cast<uint32_t>(sp));
#pragma unroll
            for (int c = 0; c < Cfg::kWgCols; c += 4) {
              const float4 t = ld_shared_cluster_f4(src + static_cast<uint32_t>(c / 4) * 512u);
              sum[c] += t.x;
              sum[c + 1] += t.y;
              sum[c + 2] += t.z;
              sum[c + 3] += t.w;
            }
          }
        }
      }
      // Rows of this warp: m_base .. m_base + 31 (lane i holds row m_base + i).
      const int64_t m_base = static_cast<int64_t>(m_blk) * Cfg::kTileM +
                             static_cast<int64_t>(rank) * kBM + quarter * 32;
      if (m_base < args.M) {
        // One copy of the slab code, not kWgSlabs: after each slab the sums
        // move down by 32 registers, so the loop body indexes statically.
#pragma unroll 1
        for (int i = 0; i < Cfg::kWgSlabs; ++i) {
          const int slab = wg + EPI * i;
          const int n0 = n_blk * BN + slab * 32;
          if ((Cfg::kSlabs % EPI == 0 || slab < Cfg::kSlabs) && n0 < args.N) {
            float(&part)[32] = *reinterpret_cast<float(*)[32]>(&sum[0]);
            epilogue_slab<F16>(args, m_base, lane, n0, part, stg, &tmap_h, &tmap_h2,
                               &res_bar[warp - 4], res_phase, ln_mu, ln_rstd);
          }
          if (i + 1 < Cfg::kWgSlabs) {
#pragma unroll
            for (int c = 0; c + 32 < Cfg::kWgCols; ++c) sum[c] = sum[c + 32];
          }
        }
      }
    }
    // TMA stores of the result complete before the CTA can exit.
    if ((args.tma_h16 || args.tma_out || args.tma_h16b) && lane == 0) bulk_wait_group<0>();
  }

  tc_fence_before();
  __syncthreads();
  // Pair: neither CTA releases TMEM / exits early. Split-K: no CTA exits while
  // the leader may still read its partial sums.
  if (PAIR || args.ksplit > 1) cluster_sync_all();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) {
      tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    } else {
      tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
  }
}

// ---------------------------------------------------------------- host side
namespace {

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    } else {
      (void)cudaGetLastError();
    }
  });
  return g_encode;
}

}  // namespace

int encode_tmap(CUtensorMap* map, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides, const uint32_t* box, int swizzle128) {
  return encode_tmap_typed(map, rank, base, dims, strides, box, swizzle128, 0);
}

int encode_tmap_typed(CUtensorMap* map, int rank, const void* base, const uint64_t* dims,
                      const uint64_t* strides, const uint32_t* box, int swizzle128, int f16) {
  auto enc = encode_fn();
  if (enc == nullptr) return VITB200_E_NO_TMA;
  if (rank < 1 || rank > 5) return VITB200_E_INVALID_ARG;
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = static_cast<cuuint64_t>(dims[i]);
    bx[i] = static_cast<cuuint32_t>(box[i]);
    es[i] = 1;
    if (i + 1 < rank) st[i] = static_cast<cuuint64_t>(strides[i]);
  }
  const CUtensorMapSwizzle sw = swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUtensorMapDataType dt = f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = enc(map, dt, static_cast<cuuint32_t>(rank),
                   const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : VITB200_E_NO_TMA;
}

// Tensor map over a TF32 pair [2][rows][Kp]: box = [2][box_rows][BK] with the
// swizzle matching a BK*4-byte row.
int make_pair_map(CUtensorMap* map, const float* pair, int64_t rows, int Kp, int box_rows,
                  int BK) {
  return make_planes_map(map, pair, rows, Kp, 2, box_rows, BK, 0);
}

// Tensor map over `planes` planes [planes][rows][Kp] of fp32 (f16 = 0) or fp16
// elements, box = all planes x box_rows x BK, swizzle of one BK-element row.
int make_planes_map(CUtensorMap* map, const void* base, int64_t rows, int Kp, int planes,
                    int box_rows, int BK, int f16) {
  const uint64_t es = f16 ? 2 : 4;
  const uint64_t dims[3] = {static_cast<uint64_t>(Kp), static_cast<uint64_t>(rows),
                            static_cast<uint64_t>(planes)};
  const uint64_t strides[2] = {static_cast<uint64_t>(Kp) * es,
                               static_cast<uint64_t>(rows) * static_cast<uint64_t>(Kp) * es};
  const uint32_t box[3] = {static_cast<uint32_t>(BK), static_cast<uint32_t>(box_rows),
                           static_cast<uint32_t>(planes)};
  return encode_tmap_typed(map, 3, base, dims, strides, box, BK * es == 128, f16);
}

namespace {

// Tile configurations 1 .. kNumVariants - 1 (with_variant below is the table);
// 0 = automatic. 1-8 take TF32 pairs, 9-15 FP16 splits (13, 14: two B planes
// with scale-input-d); a forced variant of the other operand kind is ignored.
constexpr int kNumVariants = 16;
struct GemmPlan {
  int variant;  // tile configuration (with_variant)
  int ksplit;   // K splits (clusters of ksplit CTAs per tile; 1 = none)
};
constexpr int kPairVariant = 6;
constexpr int kF16PairVariant = 15;
// Process-wide switches and per-device caches; atomic, since host threads
// (one per GPU, say) may launch concurrently.
std::atomic<int> g_forced_variant{0};
// Split-K of small single-CTA launches (on unless switched off), and a forced
// split (0 = the cost model's choice).
std::atomic<int> g_split_k{1};
std::atomic<int> g_forced_split{0};

// Cluster-of-two slots that fit on the device at once, per device (0 = not
// queried yet).
std::atomic<int> g_pair_slots[64] = {};

constexpr int kMaxSplit = 8;  // portable cluster size

// Clusters of `d` CTAs of this kernel that fit on the device at once (cached
// per device and d; 0 when the query fails).
template <typename Kernel>
int split_cluster_slots(Kernel kernel, int smem, int threads, int d) {
  static std::atomic<int> cache[64][kMaxSplit + 1] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    (void)cudaGetLastError();
    return 0;
  }
  std::atomic<int>& slot = cache[dev][d];
  if (slot.load(std::memory_order_relaxed) == 0) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(d);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(d * (device_num_sms() / d)));
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = -1;
    }
    slot.store(n, std::memory_order_relaxed);
  }
  const int v = slot.load(std::memory_order_relaxed);
  return v > 0 ? v : 0;
}

// Whether a single-CTA launch of `tiles` output tiles over num_kb K blocks can
// split K d ways: d divides num_kb, tiles * d CTAs fit in one wave of SMs and
// all `tiles` clusters of d CTAs are resident at once.
template <typename Kernel>
bool split_fits(Kernel kernel, int smem, int threads, int64_t tiles, int num_kb, int d) {
  if (d == 1) return true;
  if (d < 1 || d > kMaxSplit || num_kb % d != 0 || tiles * d > device_num_sms()) return false;
  return split_cluster_slots(kernel, smem, threads, d) >= tiles;
}

template <int KIND, int BN, int BK, int STAGES, int CHUNK_KB, bool PAIR, int EPI = 2>
int launch_variant(const GemmProblem& p, int ksplit, int* err, cudaStream_t s) {
  using Cfg = GemmCfg<KIND, BN, BK, STAGES, CHUNK_KB, PAIR, EPI>;
  constexpr int kThreads = EpiCfg<EPI>::kThreads;
  constexpr bool F16 = Cfg::F16;
  CUtensorMap ta, tb;
  int st = F16 ? make_planes_map(&ta, p.a_h16, p.M, p.Kp, 2, kBM, BK, 1)
               : make_pair_map(&ta, p.a_pair, p.M, p.Kp, kBM, BK);
  if (st) return st;
  // Weights hold three planes; scale-input-d reads only the first two.
  st = F16 ? make_planes_map(&tb, p.b_h16, p.N, p.Kp, Cfg::kBPlanes, Cfg::kBRows, BK, 1)
           : make_pair_map(&tb, p.b_pair, p.N, p.Kp, Cfg::kBRows, BK);
  if (st) return st;
  GemmArgs a;
  a.M = p.M;
  a.N = p.N;
  a.Kp = p.Kp;
  a.num_n_tiles = (p.N + BN - 1) / BN;
  const int64_t m_tiles = (p.M + Cfg::kTileM - 1) / Cfg::kTileM;
  const int64_t tiles = m_tiles * a.num_n_tiles;
  if (tiles > 0x7fffffff) return VITB200_E_UNSUPPORTED;
  a.num_tiles = static_cast<int>(tiles);
  a.num_kb = (p.Kp + BK - 1) / BK;
  // Small problems (batch-1 latency) split K over clusters of CTAs so that
  // more SMs stream the operands (single-CTA tiles only).
  if (ksplit < 1 || (PAIR && ksplit != 1) || a.num_kb % ksplit != 0) return VITB200_E_INVALID_ARG;
  a.ksplit = ksplit;
  a.kb_per = a.num_kb / ksplit;
  a.num_chunks = (a.kb_per + CHUNK_KB - 1) / CHUNK_KB;
  const GemmEpilogue& e = p.epi;
  a.vec_out = (e.out != nullptr) && (reinterpret_cast<uintptr_t>(e.out) % 16 == 0) &&
              (e.ldo % 4 == 0) && (e.mode != kModeSplit3 || e.split_plane % 4 == 0);
  a.vec_pair = (e.out_pair != nullptr) && (reinterpret_cast<uintptr_t>(e.out_pair) % 16 == 0) &&
               (e.ldp % 4 == 0) && (e.pair_plane % 4 == 0);
  a.vec_res = (e.residual != nullptr) && (reinterpret_cast<uintptr_t>(e.residual) % 16 == 0) &&
              (e.ldr % 4 == 0);
  a.vec_h16 = (e.out_h16 != nullptr) && (reinterpret_cast<uintptr_t>(e.out_h16) % 16 == 0) &&
              (e.ldh % 8 == 0) && (e.h16_plane % 8 == 0);
  // The accumulator holds 2^11 * s * (A.B) (three-plane kind) or s * (A.B)
  // (scale-input-d), s the scale B was split with; p.acc_scale = 2^-11 / s.
  a.acc_scale = F16 ? (Cfg::SD ? p.acc_scale * kH16LoScale : p.acc_scale) : 1.f;
  a.vec_bias = (e.bias != nullptr) && (reinterpret_cast<uintptr_t>(e.bias) % 16 == 0);
  a.err = err;
  a.epi = e;
  // FP16 splits written through TMA tensor stores from the transpose buffers
  // (box {32 columns, 32 rows, 2 planes}, 64-byte swizzle): the split as the
  // only output (fc1's H), and the q and k splits of the QKV epilogue when k16
  // directly follows q16's two planes.
  CUtensorMap th, th2;
  std::memset(&th, 0, sizeof(th));
  std::memset(&th2, 0, sizeof(th2));
  a.tma_h16 = 0;
  a.tma_out = 0;
  a.tma_h16b = 0;
  if (tma_store_enabled()) {
    const uint32_t box[3] = {32, 32, 2};
    if (e.out_h16 != nullptr && a.vec_h16 && e.out == nullptr && e.out_pair == nullptr &&
        e.residual == nullptr && e.mode == kModePlain && p.N % 32 == 0) {
      const uint64_t dims[3] = {static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.M), 2};
      const uint64_t strides[2] = {static_cast<uint64_t>(e.ldh) * 2,
                                   static_cast<uint64_t>(e.h16_plane) * 2};
      if (int st2 = encode_tmap_typed(&th, 3, e.out_h16, dims, strides, box, 0, 1)) return st2;
      a.tma_h16 = 1;
    } else if (e.mode == kModeQKVAttn16 && e.k16 == e.q16 + 2 * p.M * e.e_split) {
      const uint64_t E = static_cast<uint64_t>(e.e_split);
      const uint64_t dims[3] = {E, static_cast<uint64_t>(p.M), 4};
      const uint64_t strides[2] = {E * 2, static_cast<uint64_t>(p.M) * E * 2};
      if (int st2 = encode_tmap_typed(&th, 3, e.q16, dims, strides, box, 0, 1)) return st2;
      a.tma_h16 = 1;
    } else if (e.out != nullptr && a.vec_out && e.out_pair == nullptr &&
               e.mode == kModePlain && p.N % 32 == 0 &&
               (e.residual == nullptr || (e.residual == e.out && e.ldr == e.ldo))) {
      // The fp32 result (and the residual it replaces), box {32 columns, 32
      // rows}: the transpose buffer's layout is the map's 128-byte swizzle;
      // an FP16 split of the same result through the second map.
      const uint64_t dims[3] = {static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.M), 1};
      const uint64_t strides[2] = {static_cast<uint64_t>(e.ldo) * 4,
                                   static_cast<uint64_t>(e.ldo) * 4 * static_cast<uint64_t>(p.M)};
      const uint32_t box32[3] = {32, 32, 1};
      if (int st2 = encode_tmap_typed(&th, 3, e.out, dims, strides, box32, 1, 0)) return st2;
      a.tma_out = 1;
      if (e.out_h16 != nullptr && a.vec_h16) {
        const uint64_t hd[3] = {static_cast<uint64_t>(p.N), static_cast<uint64_t>(p.M), 2};
        const uint64_t hs[2] = {static_cast<uint64_t>(e.ldh) * 2,
                                static_cast<uint64_t>(e.h16_plane) * 2};
        if (int st2 = encode_tmap_typed(&th2, 3, e.out_h16, hd, hs, box, 0, 1)) return st2;
        a.tma_h16b = 1;
      }
    }
  }
  if constexpr (PAIR) {
    int dev = 0;
    if (int st2 = cuda_status(cudaGetDevice(&dev))) return st2;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int slots = (dev >= 0 && dev < 64) ? g_pair_slots[dev].load(std::memory_order_relaxed) : 0;
    if (slots <= 0) {
      cfg.gridDim = dim3(2 * static_cast<unsigned>(device_num_sms() / 2));
      if (cudaOccupancyMaxActiveClusters(&slots, gemm_tf32x3_kernel<KIND, BN, BK, STAGES, CHUNK_KB, PAIR, EPI>,
                                         &cfg) != cudaSuccess ||
          slots <= 0) {
        (void)cudaGetLastError();
        slots = device_num_sms() / 2;
      }
      if (dev >= 0 && dev < 64) g_pair_slots[dev].store(slots, std::memory_order_relaxed);
    }
    const dim3 grid(2 * static_cast<unsigned>(std::min<int64_t>(tiles, slots)));
    st = launch_kernel(gemm_tf32x3_kernel<KIND, BN, BK, STAGES, CHUNK_KB, PAIR, EPI>, grid,
                       dim3(kThreads), Cfg::kSmemBytes, s, 2, ta, tb, th, th2, a);
    if (st) return st;
    return cuda_status(cudaGetLastError());
  } else {
    // Split: exactly one CTA per (tile, split), clusters of ksplit CTAs.
    const dim3 grid(static_cast<unsigned>(
        a.ksplit > 1 ? tiles * a.ksplit : std::min<int64_t>(tiles, device_num_sms())));
    st = launch_kernel(gemm_tf32x3_kernel<KIND, BN, BK, STAGES, CHUNK_KB, PAIR, EPI>, grid,
                       dim3(kThreads), Cfg::kSmemBytes, s, static_cast<unsigned>(a.ksplit), ta,
                       tb, th, th2, a);
    if (st) return st;
    return cuda_status(cudaGetLastError());
  }
}

template <int KIND, int BN, int BK, int STAGES, int CHUNK_KB, bool PAIR, int EPI = 2>
int set_smem_attr() {
  using Cfg = GemmCfg<KIND, BN, BK, STAGES, CHUNK_KB, PAIR, EPI>;
  return cuda_status(cudaFuncSetAttribute(gemm_tf32x3_kernel<KIND, BN, BK, STAGES, CHUNK_KB, PAIR, EPI>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          Cfg::kSmemBytes));
}

// A tile configuration as a type, for visitors over the variant table.
template <int KIND_, int BN_, int BK_, int STAGES_, int CHUNK_KB_, bool PAIR_, int EPI_ = 2>
struct VariantT {
  static constexpr int KIND = KIND_, BN = BN_, BK = BK_, STAGES = STAGES_, CHUNK_KB = CHUNK_KB_;
  static constexpr bool PAIR = PAIR_;
  static constexpr int EPI = EPI_;
  using Cfg = GemmCfg<KIND, BN, BK, STAGES, CHUNK_KB, PAIR, EPI>;
  static constexpr auto kernel() {
    return gemm_tf32x3_kernel<KIND, BN, BK, STAGES, CHUNK_KB, PAIR, EPI>;
  }
};

// The table of tile configurations: calls f(VariantT<...>{}) for variant v
// (1 .. kNumVariants - 1).
template <typename F>
int with_variant(int v, F&& f) {
  switch (v) {
    case 1: return f(VariantT<kKindTF32, 128, 32, 2, 4, false>{});
    case 2: return f(VariantT<kKindTF32, 128, 16, 5, 8, false>{});
    case 3: return f(VariantT<kKindTF32, 64, 32, 3, 4, false>{});
    case 4: return f(VariantT<kKindTF32, 128, 32, 2, 2, false>{});
    case 5: return f(VariantT<kKindTF32, 256, 16, 3, 8, false>{});
    case 6: return f(VariantT<kKindTF32, 256, 32, 2, 4, true>{});
    case 7: return f(VariantT<kKindTF32, 256, 16, 5, 8, true>{});
    case 8: return f(VariantT<kKindTF32, 256, 16, 5, 16, true>{});
    case 9: return f(VariantT<kKindF16, 256, 64, 2, 2, true>{});
    case 10: return f(VariantT<kKindF16, 128, 64, 2, 2, false>{});
    case 11: return f(VariantT<kKindF16, 64, 64, 3, 2, false>{});
    case 12: return f(VariantT<kKindF16, 256, 32, 4, 4, true>{});
    case 13: return f(VariantT<kKindF16SD, 256, 64, 2, 1, true>{});
    case 14: return f(VariantT<kKindF16SD, 128, 64, 2, 1, false>{});
    case 15: return f(VariantT<kKindF16, 256, 64, 2, 4, true>{});
    default: return VITB200_E_UNSUPPORTED;
  }
}

// Launch cost model for small problems, in units of about 40 ps. A CTA's K
// loop is latency-bound (a few stages of operands in flight per SM), so a K
// block costs about (stage bytes) / (stages): measured on B200 at M = 197,
// 0.75 us for 64-wide F16 tiles (3 stages of 56 KB), 1.5 us for 128-wide ones
// (2 of 80 KB). A split adds the cluster barriers and the leader's reads of
// the partial tiles over distributed shared memory (under 1 us at d = 4).
constexpr int64_t kSplitFixedCost = 12 * 1024;
constexpr int64_t kSplitPerCtaCost = 5 * 1024;

// Tile configuration and K split of a launch. Large problems (M >= 1024):
// 256 x 128 tiles on CTA pairs (each SM streams half of B, so operand traffic
// per FLOP matches a 256-wide tile), no split. Small ones (batch-1 latency):
// among the single-CTA tile widths and the K splits that fit, the cheapest by
// the model above: (waves) x (K blocks per split) x (cost of a K block) + the
// split's cost; a partial last wave costs a full one.
GemmPlan plan_gemm(int64_t M, int N, int Kp, bool f16) {
  GemmPlan plan{0, 1};
  const int forced = g_forced_variant;
  const bool use_forced =
      forced != 0 &&
      with_variant(forced, [](auto t) { return int{decltype(t)::KIND != kKindTF32}; }) == f16;
  if (!use_forced && M >= 1024) {
    plan.variant = f16 ? kF16PairVariant : kPairVariant;
    return plan;
  }
  const int sms = device_num_sms();
  const int64_t m_tiles = (M + kBM - 1) / kBM;
  const int cands_f16[2] = {10, 11}, cands_tf32[2] = {1, 3};  // BN = 128, 64
  const int* cands = f16 ? cands_f16 : cands_tf32;
  int64_t best_cost = 0;
  bool have = false;
  const int forced_d = g_split_k ? g_forced_split.load() : 0;
  for (int i = 0; i < (use_forced ? 1 : 2); ++i) {
    const int v = use_forced ? forced : cands[i];
    with_variant(v, [&](auto t) {
      using T = decltype(t);
      const int64_t tiles = (T::PAIR ? (M + 2 * kBM - 1) / (2 * kBM) : m_tiles) *
                            ((N + T::BN - 1) / T::BN);
      const int num_kb = (Kp + T::BK - 1) / T::BK;
      const int max_d = (T::PAIR || !g_split_k) ? 1 : kMaxSplit;
      for (int d = 1; d <= max_d; ++d) {
        if (!split_fits(T::kernel(), T::Cfg::kSmemBytes, EpiCfg<T::EPI>::kThreads, tiles, num_kb,
                        d))
          continue;
        const int64_t waves = (tiles * d + sms - 1) / sms;
        int64_t cost = waves * (num_kb / d) * (T::Cfg::kStageBytes / T::STAGES) +
                       (d > 1 ? kSplitFixedCost + (d - 1) * kSplitPerCtaCost : 0);
        // A forced split that fits wins over every other choice.
        if (forced_d > 0 && d == forced_d) cost -= int64_t{1} << 40;
        if (!have || cost < best_cost) {
          have = true;
          best_cost = cost;
          plan.variant = v;
          plan.ksplit = d;
        }
      }
      return 0;
    });
  }
  return plan;
}

}  // namespace

int gemm_set_split_k(int enable) {
  const int old = g_split_k.exchange(enable != 0 ? 1 : 0);
  return old;
}

int gemm_set_split(int d) {
  const int old = g_forced_split.load();
  if (d >= 0 && d <= kMaxSplit) g_forced_split.store(d);
  return old;
}

int gemm_set_variant(int v) {
  const int old = g_forced_variant.load();
  if (v >= 0 && v < kNumVariants) g_forced_variant.store(v);
  return old;
}

int gemm_prepare_device() {
  for (int v = 1; v < kNumVariants; ++v) {
    const int st = with_variant(v, [](auto t) {
      using T = decltype(t);
      return set_smem_attr<T::KIND, T::BN, T::BK, T::STAGES, T::CHUNK_KB, T::PAIR, T::EPI>();
    });
    if (st) return st;
  }
  if (encode_fn() == nullptr) return VITB200_E_NO_TMA;
  return 0;
}

int gemm_pairs_launch(const GemmProblem& p, cudaStream_t s) {
  const bool f16 = p.f16 != 0;
  if (p.M < 0 || p.N < 0 || p.Kp < 0 || (p.Kp % (f16 ? 8 : 4)) != 0) return VITB200_E_INVALID_ARG;
  if (p.epi.out == nullptr && p.epi.out_pair == nullptr && p.epi.out_h16 == nullptr &&
      p.epi.mode != kModeQKVAttn16)
    return VITB200_E_INVALID_ARG;
  if (p.M == 0 || p.N == 0) return 0;
  if (p.epi.mode == kModeSplit3 && (p.epi.e_split <= 0 || p.epi.e_split % 32 != 0))
    return VITB200_E_UNSUPPORTED;
  if (p.epi.mode == kModeQKVAttn &&
      (p.epi.e_split <= 0 || p.epi.e_split % 64 != 0 || p.N != 3 * p.epi.e_split ||
       !p.epi.vt_pair || !p.epi.out_pair || p.epi.out || p.epi.residual || p.epi.T <= 0 ||
       p.epi.T4 < p.epi.T || p.epi.ldp != 2 * p.epi.e_split))
    return VITB200_E_INVALID_ARG;
  if (p.epi.mode == kModePatch && (p.epi.P <= 0 || p.epi.T != p.epi.P + 1 || !p.epi.pos))
    return VITB200_E_INVALID_ARG;
  if (p.epi.mode == kModeQKVAttn16 &&
      (p.epi.e_split <= 0 || p.epi.e_split % 64 != 0 || p.N != 3 * p.epi.e_split ||
       !p.epi.q16 || !p.epi.k16 || !p.epi.vt16 || p.epi.out || p.epi.out_pair || p.epi.out_h16 ||
       p.epi.residual || p.epi.gelu || p.epi.T <= 0 || p.epi.T4 < p.epi.T || p.epi.T4 % 8 ||
       reinterpret_cast<uintptr_t>(p.epi.q16) % 16 || reinterpret_cast<uintptr_t>(p.epi.k16) % 16))
    return VITB200_E_INVALID_ARG;
  // Folded LayerNorm and row statistics: whole 32-column slabs, written by the
  // staged epilogue (16-byte aligned rows).
  if (p.epi.ln_c != nullptr && (!p.epi.ln_d || !p.epi.ln_stats || p.epi.ln_slabs <= 0 ||
                                p.epi.ln_slabs > kMaxLnSlabs || p.epi.bias || p.Kp == 0))
    return VITB200_E_INVALID_ARG;
  if (p.epi.stats_out != nullptr &&
      (p.N % 32 || !p.epi.out || reinterpret_cast<uintptr_t>(p.epi.out) % 16 || p.epi.ldo % 4 ||
       (p.epi.residual && (reinterpret_cast<uintptr_t>(p.epi.residual) % 16 || p.epi.ldr % 4)) ||
       (p.epi.out_h16 && (reinterpret_cast<uintptr_t>(p.epi.out_h16) % 16 || p.epi.ldh % 8 ||
                          p.epi.h16_plane % 8)) ||
       p.epi.out_pair || p.epi.mode != kModePlain || p.Kp == 0))
    return VITB200_E_UNSUPPORTED;
  if (p.Kp == 0) return gemm_k0_launch(p, s);
  const void* a_ptr = f16 ? static_cast<const void*>(p.a_h16) : p.a_pair;
  const void* b_ptr = f16 ? static_cast<const void*>(p.b_h16) : p.b_pair;
  if (a_ptr == nullptr || b_ptr == nullptr) return VITB200_E_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(a_ptr) % 16 || reinterpret_cast<uintptr_t>(b_ptr) % 16)
    return VITB200_E_ALIGNMENT;
  int* err = device_error_word();
  if (err == nullptr) return VITB200_E_INVALID_ARG;
  const GemmPlan plan = plan_gemm(p.M, p.N, p.Kp, f16);
  return with_variant(plan.variant, [&](auto t) {
    using T = decltype(t);
    return launch_variant<T::KIND, T::BN, T::BK, T::STAGES, T::CHUNK_KB, T::PAIR, T::EPI>(
        p, plan.ksplit, err, s);
  });
}

int gemm_plan(int64_t M, int N, int Kp, int f16, int* variant, int* ksplit) {
  if (M <= 0 || N <= 0 || Kp <= 0) return VITB200_E_INVALID_ARG;
  const GemmPlan plan = plan_gemm(M, N, Kp, f16 != 0);
  if (variant) *variant = plan.variant;
  if (ksplit) *ksplit = plan.ksplit;
  return 0;
}

}  // namespace vitb200
