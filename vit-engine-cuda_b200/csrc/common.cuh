// Device-side helpers shared by the sm_100a kernels of libvitb200.so:
// TF32 hi/lo splitting, bounded mbarrier waits, TMA, tcgen05/TMEM wrappers.
//
// Every wait on an mbarrier is bounded: after kWaitTimeoutNs of polling (or as
// soon as another thread of the grid has already reported an error) it records
// a code in the device error word and returns false, so a kernel that lost a
// producer or consumer ends instead of hanging the GPU.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vitb200 {

// Codes written to the device error word (first writer wins).
enum DeviceError : int {
  kErrNone = 0,
  kErrWaitFull = 1,     // MMA issuer waited too long for a TMA stage
  kErrWaitEmpty = 2,    // TMA producer waited too long for a free stage
  kErrWaitAccFull = 3,  // epilogue waited too long for an accumulator
  kErrWaitAccEmpty = 4, // MMA issuer waited too long for a drained accumulator
  kErrDrain = 5,        // error path: in-flight copies did not land in time
  kErrF16Range = 6,     // a value outside the FP16-split range reached a split
  kErrWaitSplit = 7,    // split-K owner waited too long for the other CTAs' partial sums
};

constexpr unsigned long long kWaitTimeoutNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Programmatic dependent launch: every kernel of this library is launched
// allowed to start before the previous grid on its stream has finished. It
// calls griddep_wait() before its first global-memory access (this returns
// once the grids it depends on have completed and their writes are visible)
// and then griddep_launch_dependents(), so the next grid's CTAs may be
// scheduled as soon as all of this grid's CTAs have started. Without the
// launch attribute both are no-ops.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void report_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

__device__ __forceinline__ bool error_raised(const int* err) {
  return err != nullptr && *reinterpret_cast<const volatile int*>(err) != 0;
}

// ---- TF32 split --------------------------------------------------------
// hi = x rounded to TF32 (round-to-nearest, ties away: cvt.rna), lo = the
// remainder x - hi (exact in fp32) rounded to TF32 the same way. Both have
// their low 13 mantissa bits clear, so the tensor core sees them exactly.
__device__ __forceinline__ float tf32_round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

__device__ __forceinline__ void tf32_split(float x, float& hi, float& lo) {
  hi = tf32_round(x);
  lo = tf32_round(__fsub_rn(x, hi));
}

// ---- FP16 split (Ootomo & Yokota, "Recovering single precision accuracy
// from Tensor Cores while surpassing the FP32 theoretical peak performance",
// IJHPCA 2022) ----------------------------------------------------------
// x ~= hi + lo * 2^-11 with hi = fp16(x) and lo = fp16((x - hi) * 2^11). The
// remainder r = x - hi is exact in fp32 and |r| <= 2^-11 |x|; scaling it by
// 2^11 before rounding keeps lo's 11 bits unless r is tiny, so
// |x - hi - lo * 2^-11| <= 2^-22 |x| + 2^-36. A GEMM then needs
// hi*hi*2^11 + hi*lo + lo*hi, which
// the tensor core takes as three f16 products into one FP32 accumulator when
// the B operand carries a third plane hi*2^11 (every product scaled by 2^11).
// Finite only for |x| < 65504; kH16Limit is the bound callers keep to.
constexpr float kH16LoScale = 2048.f;
constexpr float kH16Limit = 32768.f;

__device__ __forceinline__ void h16_split(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(__fmul_rn(__fsub_rn(x, __half2float(hi)), kH16LoScale));
}

// The FP16 splits of two values at once, packed as they are stored (a in the
// low half, b in the high half): same rounding as h16_split, with the paired
// f32 -> f16x2 conversions.
__device__ __forceinline__ void h16_split2(float a, float b, uint32_t& hi2, uint32_t& lo2) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn(__fmul_rn(__fsub_rn(a, hf.x), kH16LoScale),
                                      __fmul_rn(__fsub_rn(b, hf.y), kH16LoScale));
  hi2 = *reinterpret_cast<const uint32_t*>(&h);
  lo2 = *reinterpret_cast<const uint32_t*>(&l);
}

// Two halves packed little-endian (column c in the low half, c+1 in the high).
__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
  return static_cast<uint32_t>(__half_as_ushort(a)) |
         (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Exact (erf) GELU, the activation of timm's ViT MLP: GELU(x) = x * Phi(x),
// Phi the standard normal CDF. Evaluated from the lower tail e = Phi(-|x|):
// GELU(x) = x - x*e for x > 0 and x*e otherwise. With a = |x|,
//   log2 Phi(-a) = g(a) - a^2 / (2 ln 2),
// where g(a) = log2(Phi(-a) e^{a^2/2}) (a scaled Mills ratio) is smooth and
// bounded (-1 at a = 0, -3.9 at a = 5.6). g is a degree-10 polynomial with
// g(0) = -1 exactly, fitted to g by weighted least squares in the Chebyshev
// basis on [0, 5.6] (the fit is reproduced by fit_gelu.py beside this file);
// beyond 5.6 the polynomial is held at g(5.6) while the a^2 term keeps
// falling, so e underflows to 0 and GELU(x) becomes x or 0. One ex2.approx and
// eleven FMAs instead of an erff call. Error against float64 GELU: relative
// <= 1e-6 for |x| < 3 (<= 2e-7 for x > 1), <= 2e-6 wherever |GELU| > 1e-6,
// absolute <= 2.4e-7
// (the final rounding of x near 8); ex2.approx adds ~2^-22 relative. NaN
// stays NaN; +-inf give NaN (inf * 0).
__device__ __forceinline__ float gelu_erf(float x) {
  const float a = fminf(fabsf(x), 5.6f);
  float h = -1.648524517e-08f;
  h = fmaf(h, a, 5.266558105e-07f);
  h = fmaf(h, a, -7.210927379e-06f);
  h = fmaf(h, a, 5.323315054e-05f);
  h = fmaf(h, a, -1.941426890e-04f);
  h = fmaf(h, a, -1.917099726e-04f);
  h = fmaf(h, a, 7.203671150e-03f);
  h = fmaf(h, a, -5.263466015e-02f);
  h = fmaf(h, a, 2.621984780e-01f);
  h = fmaf(h, a, -1.151113629e+00f);
  const float g = fmaf(h, a, -1.f);
  const float e = ex2_approx(fmaf(x * x, -0.72134752044448170368f, g));  // 1/(2 ln 2)
  const float y = x * e;
  return x > 0.f ? x - y : y;
}

// ---- shared memory / mbarrier -----------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes initialised barriers visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(addr), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase with the given parity to complete. Returns false
// (after recording `code`) on timeout or when another thread already failed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  const uint32_t addr = smem_addr(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t polls = 0;
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if ((++polls & 63u) == 0) {
      if (error_raised(err)) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        report_error(err, code);
        return false;
      }
    }
  }
}

// ---- TMA ---------------------------------------------------------------
// 3-D tiled bulk-tensor load global -> shared (this CTA only),
// completion signalled on `bar` via complete_tx.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int c0,
                                            int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 4-D variant (used for the per-head transposed V pairs).
__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, uint64_t* bar, int c0,
                                            int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 3-D tiled bulk-tensor store shared -> global (this GPU's memory), tracked by
// the issuing thread's bulk async-group. The tensor map clips rows and columns
// past its extents.
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* src, int c0, int c1,
                                             int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];"
               ::"l"(tmap), "r"(smem_addr(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N of this thread's bulk async-groups still read their
// shared-memory source (.read) or are incomplete (no .read).
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- tcgen05 / TMEM ----------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::tf32, one CTA.
__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] = A * B + D * 2^-11 (tcgen05.mma's scale-input-d): folds a product
// into an accumulator that so far holds values scaled by 2^11. kind::f16,
// operands in shared memory; one CTA, or a CTA pair.
__device__ __forceinline__ void umma_f16_sd11(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, 1, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p, 11;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc)
      : "memory");
}
__device__ __forceinline__ void umma_f16_pair_sd11(uint32_t d_tmem, uint64_t a_desc,
                                                   uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, 1, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p, 11;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc)
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (both operands f16), one CTA.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i receives lane (base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 consecutive 32-bit columns: thread i receives lane (base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Per-warpgroup register reallocation (all four warps of a warpgroup execute
// it). The caller keeps the sum over warpgroups within the block's launch
// allocation.
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// ---- UMMA descriptors ----------------------------------------------------
// Instruction descriptor, kind::tf32: A and B TF32 (format 2), D fp32
// (format 1), both operands K-major, shape M x N.
__host__ __device__ constexpr uint32_t make_idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t(N) >> 3) << 17) |
         ((uint32_t(M) >> 4) << 24);
}

// kind::f16 instruction descriptor: FP32 accumulator, A and B both f16
// (format 0), both K-major, no negation or sparsity.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t(N) >> 3) << 17) | ((uint32_t(M) >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with the
// swizzle whose row length is `row_bytes` (128 -> SWIZZLE_128B, 64 -> 64B):
// rows of row_bytes, 8-row swizzle atoms stacked every 8*row_bytes (SBO).
// The tile base must be aligned to the atom (8*row_bytes). Version 1 (sm_100).
__device__ __forceinline__ uint64_t make_sdesc_kmajor(uint32_t saddr, int row_bytes) {
  const uint64_t layout = (row_bytes == 128) ? 2ull : (row_bytes == 64 ? 4ull : 6ull);
  const uint64_t sbo = uint64_t(8 * row_bytes) >> 4;
  return uint64_t((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (sbo << 32) | (1ull << 46) |
         (layout << 61);
}

}  // namespace vitb200

namespace vitb200 {

// D[tmem] (+)= A[tmem] * B[smem desc], kind::tf32, one CTA. A (M x K, K-major)
// is read from TMEM: lane = row, one 32-bit column per K element.
__device__ __forceinline__ void umma_tf32_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16 (both f16), one CTA. A (M x K)
// is read from TMEM: lane = row, two consecutive K elements per 32-bit column
// (element k in the low half), so one MMA's K = 16 spans 8 columns.
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] = A[tmem] * B[smem desc] + D * 2^-11 (scale-input-d), kind::f16, one CTA.
__device__ __forceinline__ void umma_f16_tmem_a_sd11(uint32_t d_tmem, uint32_t a_tmem,
                                                     uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, 1, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p, 11;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from registers: thread i writes lane (base+i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

}  // namespace vitb200

namespace vitb200 {

// ---- CTA pairs (cluster of two, tcgen05 cta_group::2) --------------------
// The two CTAs of a cluster share one 256-row MMA tile; rank 0 issues the MMAs.
// Every load below is a plain per-CTA copy into the issuing CTA.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// All threads of both CTAs.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

// shared::cluster address of the object at shared::cta address `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// Bounded wait, with acquire at cluster scope, on a barrier of this CTA that
// threads of other CTAs of the cluster arrive on (mbar_arrive_cluster): their
// writes before the arrival are visible to this thread afterwards.
__device__ __forceinline__ bool mbar_try_wait_acq_cluster(uint32_t addr, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(addr), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait_acq_cluster(uint64_t* bar, uint32_t parity, int* err,
                                                      int code) {
  const uint32_t addr = smem_addr(bar);
  if (mbar_try_wait_acq_cluster(addr, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t polls = 0;
  while (true) {
    if (mbar_try_wait_acq_cluster(addr, parity)) return true;
    if ((++polls & 63u) == 0) {
      if (error_raised(err)) return false;
      if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
        report_error(err, code);
        return false;
      }
    }
  }
}

// 16-byte load from another CTA's shared memory (shared::cluster address).
__device__ __forceinline__ float4 ld_shared_cluster_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

// Orders this thread's earlier async-proxy (TMA / tensor core) accesses of
// shared memory with its later generic ones.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 3-D tiled load into this CTA's shared memory whose completion is counted on
// the mbarrier at a shared::cluster address (the pair leader's barrier).
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const void* tmap, uint32_t mbar_cluster,
                                                 int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(mbar_cluster), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D (+)= A * B^T over the CTA pair (M = 256: rows 0..127 from rank 0's shared
// memory and TMEM, 128..255 from rank 1's; B split by N the same way).
__device__ __forceinline__ void umma_tf32_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f16 on a CTA pair (A rows split across the two CTAs, B columns too).
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on the mbarrier at a shared::cluster address (either CTA of the pair)
// once the pair MMAs issued so far by this thread are done.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar_cluster) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          bar_cluster)
      : "memory");
}

}  // namespace vitb200
