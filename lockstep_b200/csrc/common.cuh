// LSSA-B8 / B9.1 contract attention for sm_100a -- shared device definitions.
//
// Contract constants (docs/contract/BLOCK_EXPONENT_VARIANT.md B8.0; reference/lssab8_golden.py:54-74).
// Every helper here is exact: integer arithmetic, or a single IEEE binary32 RNE operation on
// exactly representable operands.  The library is built with -ftz=false -prec-div=true
// -prec-sqrt=true -fmad=false so no compiler contraction or flush can change a rounding.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace lssab8 {

constexpr int kBHI = 26;          // one doubling = 2^26 in the chain
constexpr int kKB = 128;          // key block (absolute positions)
constexpr int kSEG = 32;          // fold segment, in blocks
constexpr int kSWIN = 32;         // exact-skip window, in doublings
constexpr int kWLOC = 9;          // block-local weight window, in doublings
constexpr int kNIDX = 7;          // index bits per doubling
constexpr int kTabLive = kWLOC << kNIDX;      // 1152 live T2 entries
constexpr int kTabPad = 8192;                  // zero-padded: a 32-bit d indexes it as d >> 19
constexpr int kIdxShift = kBHI - kNIDX;        // 19

// status / device error bits (the device error word is OR-accumulated)
enum : int {
  kOk = 0,
  kErrArg = 1,            // bad shape / stride / dtype / null pointer
  kErrUnsupported = 2,    // valid contract input the kernels do not cover (e.g. dh not 64/128)
  kErrCuda = 3,           // CUDA runtime error
  kErrWorkspace = 4,      // caller workspace too small
  kErrDevice = 5,         // the device error word is nonzero (see kDev*)
};
enum : int {
  kDevEvRange = 1,        // e_v outside [-32, 40] (reference/lssab9_torch.py:158)
  kDevTimeout = 2,        // a bounded wait gave up (pipeline stalled)
  kDevBadPage = 4,        // block table entry out of range
  kDevAlign = 8,          // a source row off the 16-byte grid a vectorised kernel needs
};

// dtype codes used across the C ABI
enum : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

template <int Dt> struct Elem;
template <> struct Elem<kF32> { using T = float; };
template <> struct Elem<kF16> { using T = __half; };
template <> struct Elem<kBF16> { using T = __nv_bfloat16; };

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// --------------------------------------------------------------------------------- PREP
// The clip-safe pow2 exponent of an amax m >= 0 (reference/contract_common.py:80-90,
// reference/lssab_torch.py:62-85): e = 7 - E(frexp), 0 for m == 0, minus one when
// m * 2^e > 127, clamped to [-32, hi].  With m = (1+f) 2^(be-127): e = 133 - be and
// m * 2^e = 64 (1+f) > 127  <=>  mantissa field > 0x7E0000.  Subnormal m gives e >= 132, which
// the clamp maps to hi, exactly as the reference's clamp does.
__device__ __forceinline__ int pow2_exponent(float m, int hi) {
  if (m == 0.0f) return 0;
  uint32_t u = __float_as_uint(m);
  int be = (int)(u >> 23) & 0xFF;
  int e = 133 - be - (int)((u & 0x7FFFFFu) > 0x7E0000u);
  e = e < -32 ? -32 : e;
  return e > hi ? hi : e;
}

// 2^e as an exact binary32, e in [-126, 127].
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// q = clamp(rint(x * 2^e), -127, 127): rint is round-half-even; x * 2^e is exact unless it
// is subnormal, in which case it rounds to zero either way.
__device__ __forceinline__ int quant8(float x, float sc) {
  float y = rintf(__fmul_rn(x, sc));
  y = fminf(fmaxf(y, -127.0f), 127.0f);
  return (int)y;
}

// ---------------------------------------------------------------------------------- FOLD
// G = g_fold(dh, clamp(sh, -7, 23)) in [1, 2^30] (reference/lssab_golden.py:158-168).
__device__ __forceinline__ uint32_t g_fold(uint32_t base, int sh) {
  sh = sh < -7 ? -7 : (sh > 23 ? 23 : sh);
  uint64_t G;
  if (sh >= 0) G = ((uint64_t)base + (sh > 0 ? (1ull << (sh - 1)) : 0ull)) >> sh;
  else G = (uint64_t)base << (-sh);
  G = G < 1 ? 1 : G;
  return (uint32_t)(G > (1ull << 30) ? (1ull << 30) : G);
}

// The contract rescale: exponent-field subtraction, +0.0 when the input is zero/subnormal or
// the result's biased exponent would be < 1 (reference/lssab8_golden.py:150-168).  D >= 0.
__device__ __forceinline__ float rescale(float x, int D) {
  uint32_t u = __float_as_uint(x);
  int e = (int)(u >> 23) & 0xFF;
  int ne = e - D;
  return (e >= 1 && ne >= 1) ? __uint_as_float((u & 0x807FFFFFu) | ((uint32_t)ne << 23)) : 0.0f;
}

// The same rescale in floating-point form, for applying one row's D to many values: flush to +0
// iff |x| < 2^(D - 126) (equivalently biased exponent - D < 1, or x zero / subnormal), else
// x * 2^-d1 * 2^-d2 with d1 + d2 = D, both products exact because the result is normal.  D == 0
// gives the identity (thr = 0, factors 1), so lanes without a rescale can share the code.
// Checked against rescale() for every finite binary32 x at D = 1, 5, 126..128, 150, 200,
// 252..254 and 1000.
struct RowRescale { float s1, s2, thr; };
__device__ __forceinline__ float pow2f_sub(int e) {            // 2^e for e in [-149, 127]
  return e >= -126 ? __uint_as_float((uint32_t)(e + 127) << 23) : __uint_as_float(1u << (e + 149));
}
__device__ __forceinline__ RowRescale row_rescale(int D) {
  RowRescale r;
  if (D <= 0) { r.s1 = 1.0f; r.s2 = 1.0f; r.thr = 0.0f; return r; }
  r.thr = D <= 253 ? __uint_as_float((uint32_t)(D + 1) << 23) : __uint_as_float(0x7F800000u);
  const int d1 = D < 126 ? D : 126;
  const int d2 = D - d1 < 127 ? D - d1 : 127;
  r.s1 = pow2f_sub(-d1);
  r.s2 = pow2f_sub(-d2);
  return r;
}
__device__ __forceinline__ float apply_rescale(float x, const RowRescale& r) {
  return fabsf(x) < r.thr ? 0.0f : __fmul_rn(__fmul_rn(x, r.s1), r.s2);
}

// Exact int -> binary32 for |a| < 2^22 without the conversion pipe: the bit pattern a + 0x4B400000
// is the float 1.5*2^23 + a (its exponent cannot change for |a| < 2^22), and subtracting
// 1.5*2^23 is exact.  Every integer the fold converts is below 2^22: |A_b| <= 4,145,280,
// l_b <= 32,640, the sink product eh0*v8 <= 32,385 (docs/contract/BLOCK_EXPONENT_VARIANT.md B8.4).
__device__ __forceinline__ float i2f_small(int a) {
  return __fsub_rn(__int_as_float(a + 0x4B400000), 12582912.0f);
}

// One fold term: fl(O + f32(A) * 2^esc).  f32(A) is exact and so is the product (its exponent
// stays in the normal range, B8.5 "Ranges"), hence RN(A*sc + O) in one fused multiply-add is the
// same single rounding as the contract's add of the exact product.
__device__ __forceinline__ float fold_term(float O, int A, float sc) {
  return __fmaf_rn(i2f_small(A), sc, O);
}

// RN(y / l) for many y sharing one divisor l, given rl = RN(1 / l) (__frcp_rn, once per row).
// Markstein's method (P. W. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990): q0 = RN(y * rl) lies within 1.5 ulp of
// y / l; one correction q1 = RN(q0 + RN(y - l * q0) * rl) lies within 1 ulp; then the remainder
// r = y - l * q1 is exact in one fused multiply-add and RN(q1 + r * rl) is the correctly
// rounded quotient (Markstein's theorem: rl correctly rounded, q1 within 1 ulp).  The argument
// needs no underflow or overflow in any step, so it is used only for |y|, |l| in
// [2^-31, 2^32) (quotient and remainder far inside the normal range); any other operand
// (zero, subnormal, tiny or huge) takes the IEEE division __fdiv_rn.
__device__ __forceinline__ bool div_window(float x) {       // 2^-31 <= |x| < 2^32 (biased exponent 96..158)
  const float ax = fabsf(x);
  return ax >= 0x1p-31f && ax < 0x1p32f;
}
__device__ __forceinline__ float div_markstein(float y, float l, float rl) {
  const float q0 = __fmul_rn(y, rl);
  const float q1 = __fmaf_rn(__fmaf_rn(-q0, l, y), rl, q0);
  return __fmaf_rn(__fmaf_rn(-q1, l, y), rl, q1);
}
__device__ __noinline__ float div_rn_ieee(float y, float l) { return __fdiv_rn(y, l); }
__device__ __forceinline__ float div_rn_shared(float y, float l, float rl) {
  if (div_window(y) && div_window(l)) return div_markstein(y, l, rl);
  return div_rn_ieee(y, l);                 // rare: kept out of line
}

// least multiple of 2^26 >= m*G, returned as NB / 2^26 (|NB| < 2^52, so it fits in int32).
__device__ __forceinline__ int nb_of(int m, uint32_t G) {
  long long sg = (long long)m * (long long)G;
  return (int)((sg + ((1ll << kBHI) - 1)) >> kBHI);
}

// Programmatic dependent launch: allow the next kernel on the stream to start launching, and
// wait for the previous kernel's completion and memory (a no-op when launched without PDL).
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------ bounded waits + PTX
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread for up to ~20 us while the phase is incomplete, so a
// waiting warp issues a handful of instructions instead of spinning.
__device__ __forceinline__ bool mbar_try_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(20000u) : "memory");
  return ok != 0;
}

// The wall-time limit of every bounded wait (ns).  A kernel may pass a shorter one (the timeout
// self-test does); nothing in a healthy pipeline waits longer than microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Bounded wait on an mbarrier phase.  Gives up after limit_ns of wall time or as soon as another
// role of the CTA has raised *abort; on giving up it records kDevTimeout in *err and returns
// false so the caller can unwind without hanging the GPU.
// sleep_ns > 0 parks the thread between polls: roles that are not on the critical path (the
// fold warps, the MMA and TMA threads) must not steal issue slots from the warps that are.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err,
                                          uint32_t sleep_ns = 0, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    if (sleep_ns) {
      // non-blocking test between naps: a suspended try_wait can sleep past a phase completed
      // by tcgen05.commit, which is how the pipelines here release their buffers
      __nanosleep(sleep_ns);
      if (mbar_test(bar, parity)) return true;
    } else if (mbar_try_suspend(bar, parity)) {
      return true;
    }
    if ((it & 15u) == 15u) {
      if (*abort) return false;
      if (globaltimer() - t0 > limit_ns) {
        *abort = 1;
        if (err) atomicOr(err, kDevTimeout);
        return false;
      }
    }
  }
}


// Non-blocking poll of an mbarrier phase (no hardware suspension: arrivals made by
// tcgen05.commit are observed as soon as they land).  Same bounds as mbar_wait.
__device__ __forceinline__ bool mbar_poll(uint64_t* bar, uint32_t parity, volatile int* abort, int* err,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_test(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    if (mbar_test(bar, parity)) return true;
    if ((it & 1023u) == 1023u) {
      if (*abort) return false;
      if (globaltimer() - t0 > limit_ns) {
        *abort = 1;
        if (err) atomicOr(err, kDevTimeout);
        return false;
      }
    }
  }
}

// Named barrier with an OR-reduction: every participant gets the same answer, so a group can
// decide to unwind together (no participant can leave while others wait at a barrier).
__device__ __forceinline__ bool bar_any(int bar_id, int nthreads, bool pred) {
  uint32_t r;
  asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n barrier.cta.red.or.pred p, %2, %3, q;\n"
               " selp.u32 %0, 1, 0, p;\n}"
               : "=r"(r) : "r"((uint32_t)pred), "r"(bar_id), "r"(nthreads) : "memory");
  return r != 0;
}

// Group wait: thread `leader` of a group of `nthreads` (whole warps) polls the phase, then the
// group meets at named barrier `bar_id`, so only one thread spins while the others are parked.
// The barrier's OR-reduction makes the give-up decision identical for every member; on success
// each member re-tests the completed phase (it cannot be reused before this group releases it)
// for its own acquire ordering.
__device__ __forceinline__ bool group_wait(uint64_t* bar, uint32_t parity, bool leader, int bar_id, int nthreads,
                                           volatile int* abort, int* err) {
  bool fail = false;
  if (leader) fail = !mbar_poll(bar, parity, abort, err);
  if (bar_any(bar_id, nthreads, fail || *abort != 0)) return false;
  (void)mbar_test(bar, parity);
  return true;
}

// Warp-uniform poll for phases completed by tcgen05.commit: lane 0 polls (bounded, abort-aware),
// the verdict is broadcast, and on success every lane observes the completed phase itself (it
// cannot advance again before this warp arrives on the matching release barrier), which gives
// each lane the acquire ordering.  Every lane returns the same value.
__device__ __forceinline__ bool warp_poll(uint64_t* bar, uint32_t parity, volatile int* abort, int* err,
                                          uint64_t limit_ns = kWaitLimitNs) {
  // common case: the phase is already complete and every lane's own test says so (one test)
  if (__all_sync(0xffffffffu, mbar_test(bar, parity))) return true;
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_poll(bar, parity, abort, err, limit_ns) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) (void)mbar_test(bar, parity);
  return ok != 0;
}

// Warp-uniform form of mbar_wait for warps that next issue .sync.aligned instructions
// (tcgen05.ld): lane 0 does the bounded wait, the verdict is broadcast, and on success every
// lane observes the completed phase itself (it cannot advance again before this warp arrives
// on the matching release barrier), which gives each lane the acquire ordering.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort, int* err,
                                               uint32_t sleep_ns = 0) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort, err, sleep_ns) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) {
    // completes on the first try by the argument above; bounded all the same
    uint32_t it = 0;
    while (!mbar_try(bar, parity) && ++it < (1u << 22)) {
    }
    if (it >= (1u << 22)) {
      *abort = 1;
      if (err) atomicOr(err, kDevTimeout);
      ok = 0;
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  return ok != 0;
}

}  // namespace lssab8
