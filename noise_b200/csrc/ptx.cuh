// Inline-PTX building blocks for sm_100a: mbarriers with bounded waits, TMA tile loads, tcgen05 (TMEM alloc,
// MMA, commit, loads) and the shared-memory / instruction descriptors of tcgen05.mma kind::f16.
//
// Every spin-wait here is bounded: after NOISE_WAIT_LIMIT_NS of global time a wait gives up, records
// NOISE_DEV_TIMEOUT in the caller's status word and returns false, and the kernels then unwind (drain, free
// TMEM, return) instead of hanging the GPU.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

#ifndef NOISE_WAIT_LIMIT_NS
#define NOISE_WAIT_LIMIT_NS 2000000000ull  // 2 s: legitimate pipeline waits are microseconds
#endif

#define NOISE_DEV_TIMEOUT 1
#define NOISE_DEV_BAD_INDEX 2

namespace noise {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
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

// Non-blocking test: has the phase of the given parity completed?
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase of the given parity to complete. Returns false (and records a timeout) if it does not
// complete within NOISE_WAIT_LIMIT_NS, or at once if another thread of the grid already recorded an error.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t start = global_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 255u) == 0) {
      if (status && *(volatile int*)status != 0) return false;
      if (global_ns() - start > NOISE_WAIT_LIMIT_NS) {
        record_error(status, NOISE_DEV_TIMEOUT);
        return false;
      }
    }
  }
}

// The whole warp waits (every lane polls the same phase) and agrees on the outcome, so the issuing warp stays
// converged: its descriptor arithmetic runs once for the warp and elect_one() predicates the issue.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* status) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, status));
}

// One lane of a converged warp (always the same one, so tcgen05.commit tracks the MMAs it issued). Issuing
// tcgen05.mma under this predicate from a warp-wide loop measured 32 cycles per 128 x 64 x 16 MMA against 55 from
// a single-thread branch.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile("{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}" : "=r"(pred));
  return pred != 0;
}

// Named barrier 1 over the NT consumer (weight / epilogue) threads of the calling kernel, returning the AND of their
// predicates (a warp whose bounded wait gave up still arrives, with false, so every warp leaves together).
template <int NT>
__device__ __forceinline__ bool bar_and(bool pred) {
  static_assert(NT % 32 == 0, "whole warps");
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, 1, %2, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "n"(NT)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), no multicast
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---------------------------------------------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------------------------------------------
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

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 operands, fp32 accumulate), issued by one thread.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::tf32: fp32 operands in shared memory of which the tensor core reads the tf32
// part (K = 8 per instruction: 32 bytes of each row, as kind::f16's 16 bf16 values).
__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T (A operand read from tensor memory).
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::tf32 with A read from tensor memory: one fp32 element per 32-bit column (K = 8 per instruction: 8
// columns), K-major.
__device__ __forceinline__ void tc_mma_ts_tf32(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all tcgen05 operations issued so far by this thread have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Ties N registers written by tcgen05.ld to the tcgen05.wait::ld before this point: the compiler sees them modified
// here, so no use of them moves above the wait (they are only valid after it).
template <int N>
__device__ __forceinline__ void reg_fence(float* v) {
#pragma unroll
  for (int i = 0; i < N; i += 8)
    asm volatile("" : "+f"(v[i]), "+f"(v[i + 1]), "+f"(v[i + 2]), "+f"(v[i + 3]), "+f"(v[i + 4]), "+f"(v[i + 5]),
                 "+f"(v[i + 6]), "+f"(v[i + 7]));
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets row (lane base + i), columns c..c+31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns store (registers -> tensor memory).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Shared-memory matrix descriptor of tcgen05.mma for a K-major operand stored in 128-byte swizzled rows (the
// layout a TMA tile load with CU_TENSOR_MAP_SWIZZLE_128B writes): 8-row core groups 1024 bytes apart (SBO),
// descriptor version 1, layout type 2 (SWIZZLE_128B). The tile base must be 1024-byte aligned; the K step inside
// the 128-byte row is applied by advancing the start address by 32 bytes per 16 bf16 values.
__device__ __forceinline__ uint64_t sdesc_kmajor_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;            // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;    // SBO: 8 rows x 128 B
  d |= static_cast<uint64_t>(1u) << 46;            // version
  d |= static_cast<uint64_t>(2u) << 61;            // SWIZZLE_128B
  return d;
}

// Same, for an MN-major operand (the N index contiguous, e.g. V stored [key][dim] used as the B operand of P.V):
// 64 bf16 (128 B) of N per swizzled row, 8-row K groups 1024 bytes apart (SBO); LBO is the byte distance between
// successive 64-wide N chunks.
__device__ __forceinline__ uint64_t sdesc_mnmajor_sw128(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B, fp32 D, dense, M x N tile.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major = false, bool b_mn_major = false) {
  return (1u << 4)                                  // D format f32
         | (1u << 7)                                // A format bf16
         | (1u << 10)                               // B format bf16
         | (static_cast<uint32_t>(a_mn_major) << 15)
         | (static_cast<uint32_t>(b_mn_major) << 16)
         | (static_cast<uint32_t>(N >> 3) << 17)
         | (static_cast<uint32_t>(M >> 4) << 24);
}

// Instruction descriptor of tcgen05.mma kind::tf32: tf32 A and B (fp32 in shared memory), fp32 D, K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------------------------------------------------------
// small numerics
// ---------------------------------------------------------------------------------------------------------------
// Round to bf16 (nearest even), result widened back to fp32: the hardware conversion.
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// The same rounding on the integer ALU pipe (round half to even on the 16 dropped bits), for a kernel whose
// conversion/exponential pipe is the busier one (the LM-head cross-entropy rounds every logit next to its two MUFU
// operations). Finite inputs (all values here are).
__device__ __forceinline__ float bf16_round_alu(float x) {
  const uint32_t u = __float_as_uint(x);
  return __uint_as_float((u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u);
}

// The tf32 part of x, rounded to nearest on the 13 dropped mantissa bits (ties away from zero): exactly
// representable in tf32, |x - tf32_hi(x)| <= 2^-11 |x| and exact in fp32, so a tf32x3 product a b ~ a_hi b_hi +
// a_hi b_lo + a_lo b_hi misses only a_lo b_lo and the tf32 part of the lo terms: about 2^-22 of |a b|. Finite x.
__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
}

// e^x - 1 for two fp32 values on the FMA / ALU pipes (no MUFU), with the relative accuracy near 0 that e^x - 1
// loses: Cody-Waite reduction x = k ln2 + r, |r| <= ln2 / 2 (ln2 split into a 17-bit head and its tail, so k ln2_hi
// is exact), the Taylor polynomial of e^r - 1 to degree 8 (truncation below 2e-10 of |r|), and e^x - 1 =
// 2^k (e^r - 1) + (2^k - 1), with 2^128 applied as 2^127 * 2. x is clamped below at -87 (e^x - 1 is -1 to fp32
// precision below -17); x above ln(FLT_MAX) gives +inf, as e^x - 1 overflows there, and NaN stays NaN.
__device__ __forceinline__ float2 expm1_f2(float2 x) {
  constexpr float L2E = 1.4426950408889634f, LN2_HI = 0.693145751953125f, LN2_LO = 1.4286068203094172e-06f;
  constexpr float MAGIC = 12582912.f;        // 1.5 * 2^23: t = x / ln2 + MAGIC holds round(x / ln2) in its low bits
  constexpr float XMAX = 88.72283172607422f;  // the largest fp32 with e^x finite
  const float2 xc = make_float2(fminf(fmaxf(x.x, -87.f), XMAX), fminf(fmaxf(x.y, -87.f), XMAX));
  const float2 t = __ffma2_rn(xc, make_float2(L2E, L2E), make_float2(MAGIC, MAGIC));
  const float2 k = __fadd2_rn(t, make_float2(-MAGIC, -MAGIC));
  float2 r = __ffma2_rn(k, make_float2(-LN2_HI, -LN2_HI), xc);
  r = __ffma2_rn(k, make_float2(-LN2_LO, -LN2_LO), r);
  float2 q = __ffma2_rn(r, make_float2(1.f / 40320.f, 1.f / 40320.f), make_float2(1.f / 5040.f, 1.f / 5040.f));
  q = __ffma2_rn(q, r, make_float2(1.f / 720.f, 1.f / 720.f));
  q = __ffma2_rn(q, r, make_float2(1.f / 120.f, 1.f / 120.f));
  q = __ffma2_rn(q, r, make_float2(1.f / 24.f, 1.f / 24.f));
  q = __ffma2_rn(q, r, make_float2(1.f / 6.f, 1.f / 6.f));
  q = __ffma2_rn(q, r, make_float2(0.5f, 0.5f));
  const float2 p = __ffma2_rn(__fmul2_rn(r, r), q, r);  // e^r - 1
  const int kx = __float_as_int(t.x) - __float_as_int(MAGIC), ky = __float_as_int(t.y) - __float_as_int(MAGIC);
  const float2 s = make_float2(__int_as_float((min(kx, 127) + 127) << 23), __int_as_float((min(ky, 127) + 127) << 23));
  float2 e = __ffma2_rn(s, p, __fadd2_rn(s, make_float2(-1.f, -1.f)));
  if (kx > 127) e.x *= 2.f;  // k = 128 (x within ln2 / 2 of the overflow): 2^k (e^r - 1) + 2^k - 1 ~ 2 (2^127 e^r)
  if (ky > 127) e.y *= 2.f;
  if (!(x.x <= XMAX)) e.x = x.x > 0.f ? __int_as_float(0x7F800000) : x.x;  // overflow to +inf; NaN stays NaN
  if (!(x.y <= XMAX)) e.y = x.y > 0.f ? __int_as_float(0x7F800000) : x.y;
  return e;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Two floats rounded to bf16 (nearest even) and packed, low half = lo: one packed conversion instruction.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

__device__ __forceinline__ uint32_t pack_bf16x2_f2(float2 v) { return pack_bf16x2(v.x, v.y); }

// The two bf16 halves of a packed pair widened back to fp32 (x = low half): exact, two integer operations.
__device__ __forceinline__ float2 unpack_bf16x2(uint32_t p) {
  return make_float2(__uint_as_float(p << 16), __uint_as_float(p & 0xFFFF0000u));
}

}  // namespace noise
