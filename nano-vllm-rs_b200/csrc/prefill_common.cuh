// Device helpers shared by the two prefill kernels (prefill.cu: a pair of
// query tiles per work item; prefill_tile.cu: one query tile): tcgen05 PTX
// wrappers, shared-memory and instruction descriptors, packed FP32 math and
// the bounded warp-wide mbarrier wait.
#pragma once

#include "internal.cuh"

namespace nvb {
namespace prefill_common {

// ------------------------------------------------------------- tcgen05 PTX
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 format: start
// address >> 4 in bits 0-13, leading byte offset >> 4 in 16-29, stride byte
// offset >> 4 in 32-45, version 1 in bits 46-47, layout type 2 in 61-63).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptors, kind::f16: FP32 accumulator, BF16 A and B, A
// K-major, M = 128, N = 128. S = Q K^T: B K-major (keys). O += P V: B
// MN-major (head dims contiguous).
constexpr uint32_t kIdescBase = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 4) << 24) | ((128u >> 3) << 17);
constexpr uint32_t kIdescS = kIdescBase;
constexpr uint32_t kIdescPV = kIdescBase | (1u << 16);

// D (+)= A B with A and B from shared memory (umma_ss) or A from TMEM
// (umma_ts); each shared-memory descriptor is passed as its (low, high)
// words. The issuer builds every descriptor once and moves between
// stages and K16 steps by adding (byte offset >> 4) to the low word: the start
// address field is bits 0-13 and shared addresses stay below 2^18, so the add
// never carries out of it. This keeps the one issuing thread, which shares
// its SMSP with two softmax warps, at a few instructions per MMA.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo, uint32_t b_hi,
                                        uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\tsetp.ne.b32 p, %6, 0;\n\t"
      "mov.b64 da, {%1, %2};\n\tmov.b64 db, {%3, %4};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi, uint32_t idesc,
                                        uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\tsetp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// Packed FP32 pairs (Blackwell f32x2 ALU forms): d = a * b + c, d = a + b.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                     float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair of inputs on the FMA pipe (x <= 128), for a share of the
// softmax beside the 16-per-clock MUFU unit. Range reduction x = n + f with
// n the nearest integer (1.5 * 2^23 rounding trick, |f| <= 1/2), a degree-4
// polynomial for 2^f fitted to minimise relative error on [-1/2, 1/2] (this
// file's own fit; max relative error 2.7e-6 in FP32), then n added to the
// exponent field with one integer multiply-add. Inputs are clamped at -125,
// so a masked key (-inf) gives 2^-125 rather than 0: ~1e-38 of a value that
// the caller's V zeroing or row statistics make irrelevant.
__device__ __forceinline__ void exp2_fma_pair(float& a, float& b) {
  const float xa = fmaxf(a, -125.0f), xb = fmaxf(b, -125.0f);
  float ta, tb, na, nb, fa, fb, pa, pb;
  add2(ta, tb, xa, xb, 12582912.0f, 12582912.0f);
  add2(na, nb, ta, tb, -12582912.0f, -12582912.0f);
  fma2(fa, fb, na, nb, -1.0f, -1.0f, xa, xb);  // f = x - round(x)
  fma2(pa, pb, 0.009570096619427204f, 0.009570096619427204f, fa, fb, 0.05591785907745361f, 0.05591785907745361f);
  fma2(pa, pb, pa, pb, fa, fb, 0.240247443318367f, 0.240247443318367f);
  fma2(pa, pb, pa, pb, fa, fb, 0.6931217908859253f, 0.6931217908859253f);
  fma2(pa, pb, pa, pb, fa, fb, 0.9999992847442627f, 0.9999992847442627f);
  a = __int_as_float(__float_as_int(ta) * 8388608 + __float_as_int(pa));  // exponent += round(x)
  b = __int_as_float(__float_as_int(tb) * 8388608 + __float_as_int(pb));
}

#define NVB_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                  "=r"(r[i + 6]), "=r"(r[i + 7])
#define NVB_W8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), \
                  "r"(r[i + 6]), "r"(r[i + 7])

// 32 consecutive FP32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : NVB_R8(0), NVB_R8(8), NVB_R8(16), NVB_R8(24)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      NVB_W8(0), NVB_W8(8), NVB_W8(16), NVB_W8(24)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      NVB_W8(0), NVB_W8(8)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
}

__device__ __forceinline__ bool page_ok(int page, int num_blocks) { return page >= 0 && page < num_blocks; }


// Every lane of the warp waits; the warp continues only if all of them saw
// the phase complete, so a timeout never splits the warp before the
// .sync.aligned TMEM instructions that follow.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, kErrPrefillWait));
}

// 16 consecutive FP32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : NVB_R8(0), NVB_R8(8)
      : "r"(taddr));
}

// Uses of a tcgen05.ld destination stay after the tcgen05.wait::ld that
// completes it: the asm statements keep their order and this ties the values.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&a)[N]) {
#pragma unroll
  for (int c = 0; c < N; ++c) asm volatile("" : "+r"(a[c]));
}

}  // namespace prefill_common
}  // namespace nvb
