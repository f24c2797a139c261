// Thin inline-PTX layer for sm_100a: mbarriers, TMA tile loads, tcgen05 (MMA, TMEM alloc,
// loads/stores, commits) and the shared-memory matrix descriptors the MMA reads.
// Every wait here is bounded (kWaitLimitNs) and reports failure to its caller.
#pragma once

#include <cuda.h>
#include "common.cuh"

namespace xsake {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
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
// Non-blocking probe (acquire on success): has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
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
// Waits for the phase with the given parity to complete.  Returns false when the wait
// ran past kWaitLimitNs or *abort became non-zero (another role gave up).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) return false;
  }
}

// Warp-uniform variant for code that continues with warp-collective instructions
// (tcgen05.ld/st): every lane gets the same answer.
__device__ __forceinline__ bool warp_mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

// Warp-uniform wait for two barrier phases (the second only if `need2`, warp-uniform): both
// probes go out before either result is used, so two satisfied waits cost about one.
__device__ __forceinline__ bool warp_mbar_wait2(uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2, bool need2,
                                                volatile int* abort) {
  const bool r1 = mbar_try_wait(b1, p1);
  const bool r2 = need2 ? mbar_try_wait(b2, p2) : true;
  bool ok = true;
  if (!r1) ok = mbar_wait(b1, p1, abort);
  if (ok && !r2) ok = mbar_wait(b2, p2, abort);
  return __all_sync(0xffffffffu, ok);
}

// Warp-uniform wait for one barrier phase and, if `need23`, two more: all probes go out before
// any result is used.
__device__ __forceinline__ bool warp_mbar_wait3(uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2, uint64_t* b3,
                                                uint32_t p3, bool need23, volatile int* abort) {
  const bool r1 = mbar_try_wait(b1, p1);
  const bool r2 = need23 ? mbar_try_wait(b2, p2) : true;
  const bool r3 = need23 ? mbar_try_wait(b3, p3) : true;
  bool ok = true;
  if (!r1) ok = mbar_wait(b1, p1, abort);
  if (ok && !r2) ok = mbar_wait(b2, p2, abort);
  if (ok && !r3) ok = mbar_wait(b3, p3, abort);
  return __all_sync(0xffffffffu, ok);
}

// One lane of a converged warp (elect.sync): lets a whole warp run the uniform control flow
// of a single-issuer role while exactly one lane issues the tcgen05 / TMA instructions.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ----------------------------------------------------------------------------- fences
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ----------------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 4-D tiled load (no multicast) into this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// Untiled bulk copy global -> this CTA's shared memory (no multicast), completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// ----------------------------------------------------------------------------- tcgen05
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

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16.  A (M=128 rows x K=16) sits in TMEM with row m
// in lane m and the bf16 pair (k, k+1) in one 32-bit column (k even in the low half), so a K=16
// slice occupies 8 consecutive columns starting at a_tmem.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

#define XSAKE_TMEM_LD32(taddr, r)                                                               \
  asm volatile(                                                                                 \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"  \
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"        \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),      \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),  \
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),           \
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),           \
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])            \
      : "r"(taddr))

#define XSAKE_TMEM_ST32(taddr, r)                                                               \
  asm volatile(                                                                                 \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"   \
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"       \
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), \
      "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]),          \
      "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]),       \
      "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),       \
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])                                            \
      : "memory")

#define XSAKE_TMEM_ST16(taddr, r)                                                               \
  asm volatile(                                                                                 \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"   \
      "%13,%14,%15,%16};" ::"r"(taddr),                                                          \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),     \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]) \
      : "memory")

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// tcgen05.wait::ld that also names the 32 destination registers of a preceding load as
// in/out operands, so the compiler cannot schedule their consumers above the wait.
#define XSAKE_TMEM_WAIT_LD32(r)                                                                 \
  asm volatile("tcgen05.wait::ld.sync.aligned;"                                                 \
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),         \
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),       \
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),   \
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),   \
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),   \
                 "+r"(r[30]), "+r"(r[31])                                                        \
               :                                                                                 \
               : "memory")
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ----------------------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor, SWIZZLE_128B layout (tiles written by TMA with
// CU_TENSOR_MAP_SWIZZLE_128B, or by threads with the same XOR pattern): rows of 128 bytes,
// 8-row groups 1024 bytes apart (stride byte offset), start address 1024-aligned up to an
// in-row byte offset.  Bits: [0,14) start>>4, [16,30) leading byte offset>>4,
// [32,46) stride byte offset>>4, [46,48) version 1, [61,64) layout 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Shared-memory matrix descriptor, SWIZZLE_32B K-major layout: rows of 32 bytes (16 bf16, one
// K=16 slice), 8-row groups `sbo_bytes` apart, the 16-byte chunk index of row r XOR (r >> 2) & 1
// (sw32_offset); start address 256-aligned.  Layout type 6 = SWIZZLE_32B; the leading byte offset
// is unused by swizzled K-major layouts.
__device__ __forceinline__ uint64_t sw32_desc(uint32_t smem_addr, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)6 << 61;
  return d;
}

// Byte offset of 16-byte chunk `chunk` (0 or 1) of row r in a SWIZZLE_32B K-major block whose
// 8-row groups are 256 bytes apart.
__host__ __device__ constexpr uint32_t sw32_offset(int r, int chunk) {
  return (uint32_t)((r >> 3) * 256 + (r & 7) * 32 + ((chunk ^ ((r >> 2) & 1)) << 4));
}

// Instruction descriptor of kind::f16 with bf16 A/B, fp32 D.
// [4,6) D format (1 = F32), [7,10) A format (1 = BF16), [10,13) B format (1 = BF16),
// [15] A major (0 = K), [16] B major (0 = K, 1 = MN), [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ----------------------------------------------------------------------------- packed fp32 math
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ uint64_t pk2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t sub2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x on the FMA/ALU pipes for a pair of inputs x <= 127, to offload the MUFU unit.
// Range reduction: j = round(x) through the 1.5*2^23 rounding constant, f = x - j in
// [-0.5, 0.5] (exact), 2^f from a cubic whose coefficients were fitted in this project by
// iteratively reweighted least squares on Chebyshev nodes (max relative error 1.0e-4, far
// below bf16's 3.9e-3 spacing), then j is added to the exponent field.  Inputs are clamped
// at -125 so the exponent stays normal; 2^-125 is negligible against the row's leading
// term of 1.
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& p0, float& p1) {
  constexpr float kC1 = 0.6932829022407532f, kC2 = 0.2422109693288803f, kC3 = 0.05500892922282219f;
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const uint64_t xv = pk2(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t rc = pk2(kRound, kRound);
  const uint64_t t = add2(xv, rc);
  const uint64_t f = sub2(xv, sub2(t, rc));
  uint64_t q = fma2(pk2(kC3, kC3), f, pk2(kC2, kC2));
  q = fma2(q, f, pk2(kC1, kC1));
  q = fma2(q, f, pk2(1.0f, 1.0f));
  float t0, t1, q0, q1;
  upk2(t, t0, t1);
  upk2(q, q0, q1);
  p0 = __int_as_float(__float_as_int(q0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(q1) + (__float_as_int(t1) << 23));
}

}  // namespace sm100
}  // namespace xsake
