// Thin inline-PTX wrappers for the sm_100a features the block-sparse attention
// kernels use: mbarriers, TMA tensor loads, tcgen05 MMA / TMEM traffic, and a
// bounded wait that turns a stuck pipeline into an error status instead of a hang.
//
// Every wait in this library goes through `bounded_wait`: it gives up after
// kWaitTimeoutNs of wall time (read from %globaltimer), records
// MOSAIC_STATUS_TIMEOUT in the caller-visible status word and raises the CTA's
// abort flag so the other roles stop waiting too. No kernel traps.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "../../include/mosaic_b200.h"

namespace mosaic {

constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s per individual wait

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the barrier phase with the given parity has completed. Gives up
// (returns false) when `abort_flag` is raised by another role or when the wait
// exceeds kWaitTimeoutNs; in the latter case it raises the flag itself and
// records MOSAIC_STATUS_TIMEOUT in `status` (which may be null).
__device__ __forceinline__ bool bounded_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                             int* status, uint64_t timeout_ns = kWaitTimeoutNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > timeout_ns) {
      *abort_flag = 1;
      if (status) atomicOr(status, MOSAIC_STATUS_TIMEOUT);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive once on `bar` when every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]   (kind::f16, bf16 in, fp32 accumulate)
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor for kind::f16 with fp32 D (PTX ISA "Instruction
// descriptor" table): D fmt bits [4,6), A fmt [7,10), B fmt [10,13) (0 = f16,
// 1 = bf16; A and B always share the type), B major bit 16, N>>3 at [17,23),
// M>>4 at [24,29).
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, bool b_mn_major, uint32_t ab_fmt) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, bool b_mn_major) {
  return make_idesc(M, N, b_mn_major, 1u);
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile whose rows
// are 128 bytes (64 bf16) and whose 8-row groups are `sbo` bytes apart. Bit 46 is
// the sm_100 descriptor version, bits [61,64) = 2 selects SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t sbo, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread.
#define MOSAIC_R32(r)                                                                                        \
  "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),           \
      "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), \
      "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),          \
      "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),          \
      "=r"(r[30]), "=r"(r[31])
#define MOSAIC_W32(r)                                                                                       \
  "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),       \
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),        \
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),       \
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : MOSAIC_R32(r)
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      MOSAIC_W32(r)
      : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Makes every later use of r[0..n) depend on this point in program order, so the
// compiler cannot hoist arithmetic on tcgen05.ld results above tcgen05.wait::ld.
template <int n>
__device__ __forceinline__ void reg_fence(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < n; ++i) asm volatile("" : "+r"(r[i]));
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// The 16-bit activation type of a launch: Act<false> = bf16 (MOSAIC_DTYPE_BF16),
// Act<true> = fp16 (MOSAIC_DTYPE_F16). Values are widened to fp32 for arithmetic
// and rounded to nearest-even when stored; `round` is that store-and-reload, the
// rounding point of a tensor op whose output has the activation type.
template <bool kF16>
struct Act;
template <>
struct Act<false> {
  using T = __nv_bfloat16;
  static constexpr uint32_t kMmaFmt = 1;  // kind::f16 operand format code
  static __device__ __forceinline__ float2 unpack(uint32_t u) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return pack_bf16x2(lo, hi); }
  static __device__ __forceinline__ float to_float(T x) { return __bfloat162float(x); }
  static __device__ __forceinline__ float from_bits(uint16_t b) { return __bfloat162float(__ushort_as_bfloat16(b)); }
  static __device__ __forceinline__ T from_float(float x) { return __float2bfloat16_rn(x); }
  static __device__ __forceinline__ uint32_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
  static __device__ __forceinline__ float round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};
template <>
struct Act<true> {
  using T = __half;
  static constexpr uint32_t kMmaFmt = 0;
  static __device__ __forceinline__ float2 unpack(uint32_t u) {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float to_float(T x) { return __half2float(x); }
  static __device__ __forceinline__ float from_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }
  static __device__ __forceinline__ T from_float(float x) { return __float2half_rn(x); }
  static __device__ __forceinline__ uint32_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
  static __device__ __forceinline__ float round(float x) { return __half2float(__float2half_rn(x)); }
};


// ---------------------------------------------------------------- single-lane issue from a converged warp
// tcgen05.mma / tcgen05.commit / TMA issued by one lane chosen with elect.sync
// inside the same asm block, so the issuing warp stays converged (issuing from a
// divergent single-lane loop costs ~3x more cycles per tcgen05.mma).
__device__ __forceinline__ void mma_ss_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}
// 2D tiled bulk tensor load global -> shared by one elected lane, completion counted on
// `bar` in bytes. x is the innermost (element) coordinate, y the row coordinate. Callers
// keep x a multiple of 64 bf16 elements (128 bytes), so the 16-byte rule always holds.
__device__ __forceinline__ void tma_load_2d_elect(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];\n\t}" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// 3D tiled load (elected lane), coordinates innermost first; x a multiple of 64 bf16.
__device__ __forceinline__ void tma_load_3d_elect(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                  int z) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];\n\t}" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_elect(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
// Bounded wait for a whole warp. Every lane polls (one instruction for the warp)
// and the verdict is a warp vote, so the warp never branches on one lane's result:
// an MMA-issuing warp whose loop held a lane-0-only poll followed by a broadcast
// issued its tcgen05.mma instructions at less than half the rate it reaches this way.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* status) {
  const bool ok = bounded_wait(bar, parity, abort_flag, status);
  return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------- packed fp32 (sm_100)
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Software 2^x on the FMA/ALU pipes, for two values at once.
// Cody-Waite style reduction x = j + f with j = rint(x) (the 1.5*2^23 shifter
// trick) and f in [-1/2, 1/2], then 2^f by a degree-3 polynomial whose
// coefficients are a relative-error minimax fit computed for this library by the
// Remez exchange algorithm (max relative error 7.5e-5, far below the 2^-9 of
// the bf16 rounding that P undergoes next), and 2^j added into the exponent
// field. x is clamped at -125 so that the exponent cannot underflow and, with
// kUpper, at 126 so that it cannot wrap past the top of the exponent field either
// (without it a score more than 127 above the caller's shift would come back as a
// tiny or negative number that no sum can flag; with it the result saturates near
// 2^126, like MUFU's +inf).
template <bool kUpper = false>
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  constexpr float kC0 = 0.99992807f, kC1 = 0.69326099f, kC2 = 0.24261112f, kC3 = 0.05517167f;
  float x0, x1;
  f2_unpack(x2, x0, x1);
  x0 = fmaxf(x0, -125.0f);
  x1 = fmaxf(x1, -125.0f);
  if (kUpper) {
    x0 = fminf(x0, 126.0f);
    x1 = fminf(x1, 126.0f);
  }
  const uint64_t xc = f2_pack(x0, x1);
  const uint64_t t = f2_add(xc, f2_pack(kShift, kShift));        // low mantissa bits hold rint(x)
  const uint64_t j = f2_add(t, f2_pack(-kShift, -kShift));       // rint(x) as a float
  const uint64_t f = f2_fma(j, f2_pack(-1.0f, -1.0f), xc);       // x - rint(x), exact
  uint64_t p = f2_fma(f, f2_pack(kC3, kC3), f2_pack(kC2, kC2));
  p = f2_fma(p, f, f2_pack(kC1, kC1));
  p = f2_fma(p, f, f2_pack(kC0, kC0));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  // (bits of t) << 23 == rint(x) << 23 modulo 2^32, because 1.5*2^23 has nine zero low bits
  const float r0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  const float r1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
  return f2_pack(r0, r1);
}

}  // namespace mosaic
