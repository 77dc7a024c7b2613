// TF32x3 GEMM on sm_100a tensor cores: Y = epilogue(A * B^T) with A = X[M][K],
// B = W[N][K] (PyTorch Linear layout), both given as TF32 hi/lo pairs.
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
//    (M=128, N=BN, K=8) — lo*hi, hi*lo, hi*hi per 8-wide K slice — into four
//    TMEM chunk accumulators (two per epilogue warpgroup); a chunk spans
//    CHUNK_KB stages (K = 128) and
//    starts from zero. The tensor core's accumulator truncates toward zero, so
//    keeping each chain short is what holds FP32-level accuracy;
//  * warps 2-5 and 6-9: two epilogue warpgroups that take alternate tiles. The
//    owner of a tile drains every chunk (tcgen05.ld, one output row per thread)
//    into an FP32 running sum in registers and frees the TMEM buffer; after the
//    last chunk it applies bias / GELU / residual / positional add and stores
//    fp32 and/or the TF32 pair the next GEMM consumes, while the other
//    warpgroup is already draining the next tile's chunks.
//
// No cluster launch and no multicast: every CTA loads its own tiles.
#include <cuda.h>
#include <cudaTypedefs.h>

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
  int num_chunks;  // chunks per tile
  int vec_out;     // fp32 output rows are 16-byte aligned (float4 stores)
  int vec_pair;    // pair rows are 16-byte aligned
  int vec_res;     // residual rows are 16-byte aligned
  int* err;
  GemmEpilogue epi;
};

constexpr int kBM = 128;
constexpr int kThreads = 320;  // 10 warps: producer, MMA, 2 x 4 epilogue
constexpr int kChunkBufs = 4;  // TMEM chunk accumulators, two per epilogue warpgroup

template <int BN, int BK, int STAGES, int CHUNK_KB>
struct GemmCfg {
  static constexpr int kAPlane = kBM * BK * 4;  // bytes of one A plane (hi or lo)
  static constexpr int kBPlane = BN * BK * 4;
  static constexpr int kStageBytes = 2 * kAPlane + 2 * kBPlane;
  static constexpr int kSmemBytes = STAGES * kStageBytes + 1024;  // + alignment slack
  static constexpr int kTmemCols = kChunkBufs * BN;
  static constexpr uint32_t kIdesc = make_idesc_tf32(kBM, BN);
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert(BK * 4 == 128 || BK * 4 == 64, "BK row must be a 64B or 128B swizzle span");
  static_assert((kTmemCols & (kTmemCols - 1)) == 0 && kTmemCols >= 32 && kTmemCols <= 512,
                "TMEM columns must be a power of two in [32, 512]");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory");
  static_assert(CHUNK_KB >= 1, "chunk");
};

// Epilogue of one output row segment of 32 columns, in place on v:
// bias -> GELU -> (positional row | column split) -> residual -> fp32 / TF32-pair stores.
// The order of additions follows the reference: residual + (acc + bias)
// (vit_cuda/model.py:48,60) and (conv + bias) + pos (pos_encoding.cu:20-26).
__device__ __forceinline__ void store_row_chunk(const GemmArgs& a, int64_t m, int n0,
                                                float (&v)[32]) {
  const GemmEpilogue& e = a.epi;
  const int N = a.N;

  if (e.bias != nullptr) {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = n0 + j;
      v[j] = v[j] + ((n < N) ? __ldg(e.bias + n) : 0.f);
    }
  }
  if (e.gelu) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
  }

  int64_t out_row = m;
  int64_t col_base = n0;
  int64_t plane_off = 0;
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
  } else if (e.mode == kModeSplit3) {
    const int plane = n0 / e.e_split;  // e_split % 32 == 0: a chunk never straddles
    plane_off = static_cast<int64_t>(plane) * e.split_plane;
    col_base = n0 - plane * e.e_split;
  } else if (e.mode == kModeQKVAttn && n0 >= 2 * e.e_split) {
    // V columns: TF32 pair of V transposed per (image, head). Lanes of a warp
    // hold consecutive rows, so each column's store is one coalesced line.
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

  const bool full = (n0 + 32 <= N);
  if (e.residual != nullptr) {
    const float* r = e.residual + out_row * e.ldr + col_base;
    if (full && a.vec_res) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 t = *reinterpret_cast<const float4*>(r + j);
        v[j] = t.x + v[j];
        v[j + 1] = t.y + v[j + 1];
        v[j + 2] = t.z + v[j + 2];
        v[j + 3] = t.w + v[j + 3];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < N) v[j] = r[j] + v[j];
    }
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
    if (full && a.vec_pair) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 h, l;
        tf32_split(v[j], h.x, l.x);
        tf32_split(v[j + 1], h.y, l.y);
        tf32_split(v[j + 2], h.z, l.z);
        tf32_split(v[j + 3], h.w, l.w);
        *reinterpret_cast<float4*>(ph + j) = h;
        *reinterpret_cast<float4*>(pl + j) = l;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (n0 + j < N) {
          float h, l;
          tf32_split(v[j], h, l);
          ph[j] = h;
          pl[j] = l;
        }
    }
  }
}

// TMEM chunk buffer of chunk j of this CTA's local tile `local`. Tiles
// alternate between the two epilogue warpgroups and each warpgroup owns two of
// the four buffers, so every buffer's barriers are waited on, phase after
// phase, by exactly one waiter (mbarrier parity cannot tell phase p from p+2).
__device__ __forceinline__ void chunk_slot(int local, int j, int num_chunks, int& buf,
                                           uint32_t& use) {
  const int group = local & 1;
  const uint32_t seq = static_cast<uint32_t>((local >> 1) * num_chunks + j);
  buf = 2 * group + static_cast<int>(seq & 1u);
  use = seq >> 1;
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

template <int BN, int BK, int STAGES, int CHUNK_KB>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_b, const GemmArgs args) {
  using Cfg = GemmCfg<BN, BK, STAGES, CHUNK_KB>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t chunk_full_bar[kChunkBufs];
  __shared__ __align__(8) uint64_t chunk_empty_bar[kChunkBufs];
  __shared__ __align__(8) uint64_t mma_done_bar;
  __shared__ uint32_t tmem_base_slot;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = args.err;

  // 1024-byte aligned ring base (swizzle atoms are 8 rows x 128 B).
  const uint32_t raw_addr = smem_addr(smem_raw);
  uint8_t* ring = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < kChunkBufs; ++b) {
      mbar_init(&chunk_full_bar[b], 1);
      mbar_init(&chunk_empty_bar[b], 4);  // one arrival per draining warp
    }
    mbar_init(&mma_done_bar, 1);
    fence_barrier_init();
    prefetch_tmap(&tmap_a);
    prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_slot;

  const int num_tiles = args.num_tiles;
  const int num_kb = args.num_kb;
  const int num_chunks = args.num_chunks;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_blk = tile / args.num_n_tiles;
        const int n_blk = tile - m_blk * args.num_n_tiles;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, err, kErrWaitEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = ring + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + 2 * Cfg::kAPlane;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageBytes);
          tma_load_3d(sa, &tmap_a, &full_bar[stage], kb * BK, m_blk * kBM, 0);
          tma_load_3d(sb, &tmap_b, &full_bar[stage], kb * BK, n_blk * BN, 0);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Let every copy this thread issued land before the CTA can exit.
      for (int s = 0; s < STAGES; ++s) {
        if (issued > s) {
          const int64_t fills = (issued - s + STAGES - 1) / STAGES;
          drain_wait(&full_bar[s], static_cast<uint32_t>((fills - 1) & 1), err);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
        for (int kb = 0; kb < num_kb; ++kb) {
          const int j = kb / CHUNK_KB;
          const bool chunk_first = (kb - j * CHUNK_KB) == 0;
          const bool chunk_last = (kb - j * CHUNK_KB) == CHUNK_KB - 1 || kb == num_kb - 1;
          int buf;
          uint32_t use;
          chunk_slot(local, j, num_chunks, buf, use);
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
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            const uint32_t koff = static_cast<uint32_t>(kk * 32);  // 8 TF32 = 32 bytes
            const uint64_t dah = make_sdesc_kmajor(a_hi + koff, BK * 4);
            const uint64_t dal = make_sdesc_kmajor(a_lo + koff, BK * 4);
            const uint64_t dbh = make_sdesc_kmajor(b_hi + koff, BK * 4);
            const uint64_t dbl = make_sdesc_kmajor(b_lo + koff, BK * 4);
            const uint32_t acc0 = (chunk_first && kk == 0) ? 0u : 1u;
            umma_tf32(d_tmem, dal, dbh, Cfg::kIdesc, acc0);  // lo * hi
            umma_tf32(d_tmem, dah, dbl, Cfg::kIdesc, 1u);    // hi * lo
            umma_tf32(d_tmem, dah, dbh, Cfg::kIdesc, 1u);    // hi * hi
          }
          umma_commit(&empty_bar[stage]);  // frees the stage once these MMAs finish
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
          if (chunk_last) umma_commit(&chunk_full_bar[buf]);
        }
      }
      // Every MMA this thread issued must finish before TMEM is released.
      umma_commit(&mma_done_bar);
      drain_wait(&mma_done_bar, 0, err);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int group = (warp - 2) >> 2;  // warpgroup 0 takes even local tiles, 1 odd
    const int quarter = warp & 3;       // TMEM lanes [32*quarter, 32*quarter + 32)
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    int local = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++local) {
      if ((local & 1) != group) continue;
      const int m_blk = tile / args.num_n_tiles;
      const int n_blk = tile - m_blk * args.num_n_tiles;
      float sum[BN];
#pragma unroll
      for (int c = 0; c < BN; ++c) sum[c] = 0.f;
      for (int j = 0; j < num_chunks; ++j) {
        int buf;
        uint32_t use;
        chunk_slot(local, j, num_chunks, buf, use);
        if (!warp_wait(&chunk_full_bar[buf], use & 1u, err, kErrWaitAccFull, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int q = 0; q < BN / 32; ++q) {
          float part[32];
          __syncwarp();
          tmem_ld_32x32b_x32(lane_base + static_cast<uint32_t>(buf * BN + q * 32), part);
#pragma unroll
          for (int c = 0; c < 32; ++c) sum[q * 32 + c] += part[c];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&chunk_empty_bar[buf]);
      }
      if (!ok) break;
      const int64_t m = static_cast<int64_t>(m_blk) * kBM + row_in_tile;
      if (m < args.M) {
#pragma unroll
        for (int q = 0; q < BN / 32; ++q) {
          const int n0 = n_blk * BN + q * 32;
          if (n0 < args.N) {
            float(&part)[32] = *reinterpret_cast<float(*)[32]>(&sum[q * 32]);
            store_row_chunk(args, m, n0, part);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
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
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, static_cast<cuuint32_t>(rank),
                   const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : VITB200_E_NO_TMA;
}

// Tensor map over a TF32 pair [2][rows][Kp]: box = [2][box_rows][BK] with the
// swizzle matching a BK*4-byte row.
int make_pair_map(CUtensorMap* map, const float* pair, int64_t rows, int Kp, int box_rows,
                  int BK) {
  const uint64_t dims[3] = {static_cast<uint64_t>(Kp), static_cast<uint64_t>(rows), 2};
  const uint64_t strides[2] = {static_cast<uint64_t>(Kp) * 4,
                               static_cast<uint64_t>(rows) * static_cast<uint64_t>(Kp) * 4};
  const uint32_t box[3] = {static_cast<uint32_t>(BK), static_cast<uint32_t>(box_rows), 2};
  return encode_tmap(map, 3, pair, dims, strides, box, BK * 4 == 128);
}

namespace {

struct Variant {
  int bn, bk, stages, chunk_kb;
};
// Index 1.. are selectable with gemm_set_variant; 0 = automatic.
constexpr Variant kVariants[] = {
    {0, 0, 0, 0}, {128, 32, 3, 4}, {128, 16, 6, 8}, {64, 32, 4, 4}, {128, 32, 3, 2},
};
constexpr int kNumVariants = sizeof(kVariants) / sizeof(kVariants[0]);
int g_forced_variant = 0;

template <int BN, int BK, int STAGES, int CHUNK_KB>
int launch_variant(const GemmProblem& p, int* err, cudaStream_t s) {
  using Cfg = GemmCfg<BN, BK, STAGES, CHUNK_KB>;
  CUtensorMap ta, tb;
  int st = make_pair_map(&ta, p.a_pair, p.M, p.Kp, kBM, BK);
  if (st) return st;
  st = make_pair_map(&tb, p.b_pair, p.N, p.Kp, BN, BK);
  if (st) return st;
  GemmArgs a;
  a.M = p.M;
  a.N = p.N;
  a.Kp = p.Kp;
  a.num_n_tiles = (p.N + BN - 1) / BN;
  const int64_t m_tiles = (p.M + kBM - 1) / kBM;
  const int64_t tiles = m_tiles * a.num_n_tiles;
  if (tiles > 0x7fffffff) return VITB200_E_UNSUPPORTED;
  a.num_tiles = static_cast<int>(tiles);
  a.num_kb = (p.Kp + BK - 1) / BK;
  a.num_chunks = (a.num_kb + CHUNK_KB - 1) / CHUNK_KB;
  const GemmEpilogue& e = p.epi;
  a.vec_out = (e.out != nullptr) && (reinterpret_cast<uintptr_t>(e.out) % 16 == 0) &&
              (e.ldo % 4 == 0) && (e.mode != kModeSplit3 || e.split_plane % 4 == 0);
  a.vec_pair = (e.out_pair != nullptr) && (reinterpret_cast<uintptr_t>(e.out_pair) % 16 == 0) &&
               (e.ldp % 4 == 0) && (e.pair_plane % 4 == 0);
  a.vec_res = (e.residual != nullptr) && (reinterpret_cast<uintptr_t>(e.residual) % 16 == 0) &&
              (e.ldr % 4 == 0);
  a.err = err;
  a.epi = e;
  const int grid = static_cast<int>(std::min<int64_t>(tiles, device_num_sms()));
  gemm_tf32x3_kernel<BN, BK, STAGES, CHUNK_KB><<<grid, kThreads, Cfg::kSmemBytes, s>>>(ta, tb, a);
  count_launch();
  return cuda_status(cudaGetLastError());
}

template <int BN, int BK, int STAGES, int CHUNK_KB>
int set_smem_attr() {
  using Cfg = GemmCfg<BN, BK, STAGES, CHUNK_KB>;
  return cuda_status(cudaFuncSetAttribute(gemm_tf32x3_kernel<BN, BK, STAGES, CHUNK_KB>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          Cfg::kSmemBytes));
}

int pick_variant(int64_t M, int N) {
  // Minimise (waves of tiles) x (tile width): per-tile time grows with BN for a
  // fixed K, and a partial last wave costs a full one. Ties go to the wider tile.
  const int sms = device_num_sms();
  const int64_t m_tiles = (M + kBM - 1) / kBM;
  int best = 1;
  int64_t best_cost = -1;
  const int cands[2] = {1, 3};  // BN = 128, 64
  for (int c : cands) {
    const int bn = kVariants[c].bn;
    const int64_t tiles = m_tiles * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + sms - 1) / sms;
    const int64_t cost = waves * bn;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = c;
    }
  }
  return best;
}

}  // namespace

int gemm_set_variant(int v) {
  const int old = g_forced_variant;
  if (v >= 0 && v < kNumVariants) g_forced_variant = v;
  return old;
}

int gemm_prepare_device() {
  int st = set_smem_attr<128, 32, 3, 4>();
  if (!st) st = set_smem_attr<128, 16, 6, 8>();
  if (!st) st = set_smem_attr<64, 32, 4, 4>();
  if (!st) st = set_smem_attr<128, 32, 3, 2>();
  if (!st && encode_fn() == nullptr) st = VITB200_E_NO_TMA;
  return st;
}

int gemm_pairs_launch(const GemmProblem& p, cudaStream_t s) {
  if (p.M < 0 || p.N < 0 || p.Kp < 0 || (p.Kp % 4) != 0) return VITB200_E_INVALID_ARG;
  if (p.epi.out == nullptr && p.epi.out_pair == nullptr) return VITB200_E_INVALID_ARG;
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
  if (p.Kp == 0) return gemm_k0_launch(p, s);
  if (p.a_pair == nullptr || p.b_pair == nullptr) return VITB200_E_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(p.a_pair) % 16 || reinterpret_cast<uintptr_t>(p.b_pair) % 16)
    return VITB200_E_ALIGNMENT;
  int* err = device_error_word();
  if (err == nullptr) return VITB200_E_INVALID_ARG;
  const int v = g_forced_variant ? g_forced_variant : pick_variant(p.M, p.N);
  switch (v) {
    case 1: return launch_variant<128, 32, 3, 4>(p, err, s);
    case 2: return launch_variant<128, 16, 6, 8>(p, err, s);
    case 3: return launch_variant<64, 32, 4, 4>(p, err, s);
    case 4: return launch_variant<128, 32, 3, 2>(p, err, s);
    default: return VITB200_E_UNSUPPORTED;
  }
}

}  // namespace vitb200
