// Shared device helpers for the sm_100a paged-attention kernels.
//
// Everything here is hand-written inline PTX for Blackwell (sm_100a):
// mbarrier phase tracking with bounded waits, TMA tensor loads
// (cp.async.bulk.tensor, no multicast), and small BF16 unpack helpers.
//
// Bounded waits: every spin on an mbarrier gives up after kWaitCycles SM
// clocks (about two seconds at the B200 boost clock), records a code in the
// device-global error word `g_nvb_device_error` and returns false, so a bug
// in a pipeline turns into a readable error instead of a hung GPU.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

namespace nvb {

// Device-side error word. 0 = no error. Host reads it with
// nvb_device_error() (api.cu) and clears it with nvb_clear_device_error().
// Defined here because the library is a single translation unit.
__device__ int g_nvb_device_error = 0;

enum DeviceError : int {
  kErrNone = 0,
  kErrDecodeFullWait = 1,     // consumer gave up waiting for a KV tile
  kErrDecodeEmptyWait = 2,    // producer gave up waiting for a free stage
  kErrPrefillWait = 3,        // a prefill pipeline wait gave up
  kErrPrefillTmem = 4,        // TMEM allocation returned an unusable address
  kErrBadPage = 5,            // reserved: a page id outside [0, num_blocks)
  kErrPrefillAlign = 6,       // prefill: dynamic shared memory base not usable for the tile layout
  kErrGatherWait = 7,         // multi-GPU gather: a peer's completion flag did not arrive in time
};

constexpr long long kWaitCycles = 4000000000LL;

__device__ __forceinline__ void record_error(int code) {
  atomicCAS(&g_nvb_device_error, 0, code);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

// Makes barrier initialisation visible to the async proxy (TMA, tensor core).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Waits for the phase with the given parity to complete. Returns false (and
// records `code`) if it did not complete within kWaitCycles.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > kWaitCycles) {
      record_error(code);
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

// 3-D tiled TMA load into this CTA's shared memory; completion is reported
// as transaction bytes on `bar`. No multicast.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* desc, uint64_t* bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 3-D tiled TMA load with the default L2 policy into a shared-memory
// address (the persistent decode's per-item query tile).
__device__ __forceinline__ void tma_load_3d_plain(uint32_t dst, const void* desc, uint64_t* bar, int c0, int c1,
                                                  int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Same, with an L2 eviction-priority hint (createpolicy result).
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const void* desc, uint64_t* bar, int c0, int c1,
                                                 int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Named barrier over `threads` threads (multiple of 32) with id 1..15.
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------- BF16
// A BF16 value is the upper half of an FP32 value, so unpacking is a shift
// (low element) or a mask (high element); both are exact.
__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ void unpack8(const uint4& v, float* f) {
  f[0] = bf16lo(v.x); f[1] = bf16hi(v.x);
  f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
  f[4] = bf16lo(v.z); f[5] = bf16hi(v.z);
  f[6] = bf16lo(v.w); f[7] = bf16hi(v.w);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Division by an invariant positive divisor d with one multiply-high, after
// Granlund and Montgomery, "Division by invariant integers using
// multiplication" (PLDI 1994), figure 4.1: with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1, n / d = (mulhi(m, n) + n) >> l for every
// 32-bit unsigned n. Integer division by a value known only at run time
// otherwise goes through the MUFU reciprocal, which the softmax of the
// attention kernels keeps saturated with exponentials.
struct FastDiv {
  uint32_t m = 1, l = 0;
  int d = 1;
  static FastDiv make(int divisor) {
    FastDiv f;
    f.d = divisor;
    while ((1ull << f.l) < uint64_t(divisor)) ++f.l;
    f.m = uint32_t(((uint64_t(1) << 32) * ((uint64_t(1) << f.l) - uint64_t(divisor))) / uint64_t(divisor) + 1);
    return f;
  }
  // n >= 0
  __device__ __forceinline__ int div(int n) const {
    return int((uint64_t(__umulhi(m, uint32_t(n))) + uint32_t(n)) >> l);
  }
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace nvb
