// Paged decode attention on tcgen05 tensor cores (sm_100a), the default for
// the paged-KV decode entry points (nvb_paged_fwd*, max_q == 1).
//
// Same contract and split-KV partial format as decode.cu (reference paths:
// kernels/kernels.cu:288-354 and the FA2 decode behind
// kernels/flash_native/flash_native.cu:61-112); this kernel moves both
// contractions onto the tensor cores with the KV tokens as the M dimension,
// so up to 16 query heads of a GQA group fit the N = 16 of one MMA (larger
// groups run as several 16-head CTAs per kv head, adjacent in the grid so
// they read each K/V tile while it is in L2):
//
//   S^T_j = K_j Q^T      M = 128 tokens, N = 16 heads, K = 128 dims
//                        A = K tile (K-major, 128B-swizzled smem, by TMA)
//                        B = Q^T [16 heads][128 dims] (K-major smem)
//   O^T  += V_j^T P^T_j  M = 128 dims, N = 16 heads, K = 128 tokens
//                        A = V tile read MN-major (dims contiguous)
//                        B = P^T [16 heads][128 tokens] (K-major smem)
//
// Both accumulators live in TMEM (S^T double-buffered, 16 columns each; O^T
// 16 columns). Four softmax warps own one TMEM lane each: a token for S^T,
// a head dimension for O^T. Per 128-token tile a thread loads its 16 scores,
// the CTA agrees on each head's running max through a 4-warp shared-memory
// exchange (lazy: the max used for scaling only moves when a head's max grows
// by more than 2^8), writes its G probabilities into P^T, and keeps per-thread
// partial row sums that are reduced once at the end. The CUDA cores do a few
// instructions per KV token, so the kernel stays HBM-bound at any SM clock.
//
// Warp roles: warp 0 streams 128-token K and V tiles (32 KB each) with 3-D
// TMA into one 3-slot ring that K and V share, in the order K0 V0 K1 V1 ...
// (both tiles have the same shared-memory layout; only the MMA descriptors
// differ), so V_{j+1} is loaded as soon as S_j frees its slot rather than
// after PV_j; warp 1 owns TMEM and issues the MMAs,
// warps 2..5 run the softmax and the epilogue. 105 KB of shared memory and 64
// TMEM columns per CTA allow two CTAs per SM. Every mbarrier is waited on
// every phase, in order, by each of its waiters, except the softmax's wait
// for a V tile, taken only on tiles with masked tokens; that slot cannot run
// two phases ahead of it, since its next load needs this tile's PV.
#include "internal.cuh"

namespace nvb {

namespace decode_mma_detail {

constexpr int kTok = 128;                 // tokens per tile (MMA M)
constexpr int kN = 16;                    // padded heads per CTA (MMA N)
constexpr int kStages = 3;                // ring slots shared by K and V tiles
constexpr int kHalf = kTok * 128;         // 128 rows x 64 BF16
constexpr int kKVBytes = 2 * kHalf;       // 32 KB tile
constexpr int kNHalf = kN * 128;          // 16 rows x 64 BF16
constexpr int kNBytes = 2 * kNHalf;       // 4 KB
constexpr int kThreads = 192;
constexpr int kTmemCols = 64;             // S^T x2 at 0 and 16, O^T at 32
constexpr int kOCol = 32;
constexpr float kLn2 = 0.693147180559945309f;
constexpr float kRescaleLog2 = 8.0f;

// kXch: per-tile exchange of the four softmax warps' maxima (two barriers,
// alternating by tile parity, so each is waited on every phase in order).
enum Bar { kFull = 0, kEmpty = kFull + kStages, kSFull = kEmpty + kStages, kSFree = kSFull + 2,
           kPFull = kSFree + 2, kODone = kPFull + 1, kXch = kODone + 1, kNumBars = kXch + 2 };
constexpr int kTmemSlotOff = kNumBars * 8;
constexpr int kExchOff = kTmemSlotOff + 16;         // float [2][4 warps][16] max exchange
constexpr int kHeadBytes = kExchOff + 2 * 4 * kN * 4;
static_assert(kHeadBytes <= 1024, "barrier block must fit below the first 1 KB boundary");
// Ring load n (K of tile n / 2 when n is even, its V when odd) uses slot
// n % kStages.
constexpr int kRingOff = 0;
constexpr int kQOff = kRingOff + kStages * kKVBytes;
constexpr int kPOff = kQOff + kNBytes;
constexpr int kTileBytes = kPOff + kNBytes;
constexpr int kSmemBytes = 1024 + kTileBytes;

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
         (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// kind::f16, FP32 accumulate, BF16 A/B, M = 128, N = 16.
constexpr uint32_t kIdescBase = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t(kN) >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescS = kIdescBase;                // A K-major, B K-major
constexpr uint32_t kIdescPV = kIdescBase | (1u << 15);  // A MN-major (V^T), B K-major

__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
}

__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

// Byte offset of element (row, col) of a [rows][128] BF16 K-major operand
// stored as two 128-byte-swizzled halves of `half_bytes` each.
__device__ __forceinline__ uint32_t sw_offset(int row, int col, int half_bytes) {
  const int half = col >> 6, c = col & 63;
  return uint32_t(half * half_bytes + row * 128 + ((((c >> 3) ^ (row & 7)) << 4) | ((c & 7) << 1)));
}

__global__ void __launch_bounds__(kThreads, 2)
    decode_mma_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap kmap_half,
                      const __grid_constant__ CUtensorMap vmap_half) {
  // The kernel after this grid on the stream, when launched with
  // programmatic stream serialization (the split-KV combine, the next
  // decode), may be scheduled now; it waits (griddepcontrol.wait) for this
  // grid to complete before it touches global memory.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  const uint32_t tile_addr = (raw_addr + kHeadBytes + 1023u) & ~1023u;
  unsigned char* tiles = smem_raw + (tile_addr - raw_addr);
  const uint32_t sbase = tile_addr;

  int cta = blockIdx.x;
  const int split = cta % p.num_splits;
  cta /= p.num_splits;
  const int hgroup = cta % p.n_hgroups;
  cta /= p.n_hgroups;
  const int kvhead = cta % p.kvh;
  const int row = cta / p.kvh;
  const int head0 = kvhead * (p.qh / p.kvh) + hgroup * kN;
  const int group = min(kN, p.qh / p.kvh - hgroup * kN);  // this CTA's heads
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_raw + kTmemSlotOff);
  float* exch = reinterpret_cast<float*>(smem_raw + kExchOff);  // [2][4][kN]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // Set-up that touches only this CTA's shared memory and TMEM: when the
  // grid is launched as a programmatic dependent of the previous kernel on
  // the stream, it overlaps that kernel's tail.
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kFull + s], 1);
      mbar_init(&bars[kEmpty + s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kSFull + s], 1);
      mbar_init(&bars[kSFree + s], 4);
    }
    mbar_init(&bars[kPFull], 4);
    mbar_init(&bars[kODone], 1);
    mbar_init(&bars[kXch], 4);
    mbar_init(&bars[kXch + 1], 4);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // The previous kernel has completed, its writes visible (this grid's
  // inputs, and for split-KV the previous combine's reads of the partials
  // this grid overwrites), before any global access below.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int len = p.lens[row];
  const bool valid = len >= 1 && (long long)len <= (long long)p.table_stride * p.block_size;
  const int n_tiles_total = valid ? (len + kTok - 1) / kTok : 0;
  const int per_split = (n_tiles_total + p.num_splits - 1) / p.num_splits;
  const int t0 = split * per_split;
  const int t1 = min(t0 + per_split, n_tiles_total);
  const int ntiles = max(0, t1 - t0);
  const long long lse_base = (long long)row * p.qh * p.max_q;

  if (ntiles == 0 || tile_addr + kTileBytes > raw_addr + kSmemBytes) {
    if (ntiles != 0 && threadIdx.x == 0) record_error(kErrPrefillAlign);
    for (int e = threadIdx.x; e < group * 128; e += blockDim.x) {
      const int g = e >> 7, d = e & 127;
      const long long rh = (long long)row * p.qh + head0 + g;
      if (p.num_splits == 1) {
        p.out[rh * 128 + d] = __float2bfloat16_rn(0.0f);
        if (d == 0 && p.lse) p.lse[lse_base + (long long)(head0 + g) * p.max_q] = -INFINITY;
      } else {
        p.out_accum[((long long)split * p.rows * p.qh + rh) * 128 + d] = 0.0f;
        if (d == 0) p.lse_accum[(long long)split * p.rows * p.qh + rh] = -INFINITY;
      }
    }
    // nothing to decode: free the TMEM allocated above
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(*tmem_slot), "r"(kTmemCols)
                   : "memory");
    }
    return;
  }

  const int* table = p.block_table + (long long)row * p.table_stride;
  if (warp >= 2) {
    // Q^T [16 heads][128 dims] (rows >= group zero) and the zero rows of P^T.
    const int t = threadIdx.x - 64;
    for (int e = t; e < kN * 16; e += 128) {
      const int g = e >> 4, chunk = e & 15;
      const uint32_t dst = sbase + kQOff + sw_offset(g, chunk * 8, kNHalf);
      if (g < group) {
        const uint4 v = *reinterpret_cast<const uint4*>(p.q + ((long long)row * p.qh + head0 + g) * 128 + chunk * 8);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                     : "memory");
      } else {
        st_shared_zero16(dst);
        st_shared_zero16(sbase + kPOff + sw_offset(g, chunk * 8, kNHalf));
      }
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      tma_prefetch_desc(&kmap_half);
      tma_prefetch_desc(&vmap_half);
      const uint64_t policy = policy_evict_first();
      for (int n = 0; n < 2 * ntiles; ++n) {
        const int token0 = (t0 + (n >> 1)) * kTok;
        const int logical = token0 / p.block_size;
        const int page = table[logical];
        const bool ok = page >= 0 && page < p.num_blocks;
        const int trow = ok ? page * p.block_size + (token0 - logical * p.block_size) : 0;
        // A sequence's last tile with at most 64 live tokens loads only its
        // first 64 rows (the rest of the slot is stale and masked: scores
        // of tokens past the length are dropped and their V rows zeroed),
        // which halves the bytes read past the end of ragged contexts.
        const bool half = len - token0 <= kTok / 2;
        const CUtensorMap* m = (n & 1) ? (half ? &vmap_half : &vmap) : (half ? &kmap_half : &kmap);
        const uint32_t tile_bytes = half ? kKVBytes / 2 : kKVBytes;
        const int slot = n % kStages;
        // The slot's previous load (n - kStages) is released by the MMA that
        // read it: S of a K tile, PV of a V tile.
        if (n >= kStages && !mbar_wait(&bars[kEmpty + slot], ((n / kStages) + 1) & 1, kErrDecodeEmptyWait)) break;
        if (ok) {
          unsigned char* d = tiles + kRingOff + slot * kKVBytes;
          mbar_arrive_expect_tx(&bars[kFull + slot], tile_bytes);
          tma_load_3d_hint(d, m, &bars[kFull + slot], 0, kvhead, trow, policy);
          tma_load_3d_hint(d + kHalf, m, &bars[kFull + slot], 64, kvhead, trow, policy);
        } else {
          mbar_arrive(&bars[kFull + slot]);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool alive = true;
      const uint32_t q_addr = sbase + kQOff, p_addr = sbase + kPOff;
      auto issue_pv = [&](int t) {
        const int n = 2 * t + 1, slot = n % kStages;
        alive = alive && mbar_wait(&bars[kPFull], t & 1, kErrDecodeFullWait);
        alive = alive && mbar_wait(&bars[kFull + slot], (n / kStages) & 1, kErrDecodeFullWait);
        if (!alive) return;
        tc_fence_after();
        const uint32_t v_addr = sbase + kRingOff + slot * kKVBytes;
#pragma unroll
        for (int kk = 0; kk < kTok / 16; ++kk) {
          // A = V^T, MN-major: 64-dim halves kHalf apart, 8-token groups 1 KB apart
          const uint64_t a = sw128_desc(v_addr + kk * 2048, kHalf, 1024);
          const uint64_t b = sw128_desc(p_addr + (kk >> 2) * kNHalf + (kk & 3) * 32, 16, 1024);
          umma(tmem + kOCol, a, b, kIdescPV, (t > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars[kEmpty + slot]);
        umma_commit(&bars[kODone]);
      };
      for (int j = 0; j < ntiles && alive; ++j) {
        const int n = 2 * j, slot = n % kStages, sb = j & 1;
        alive = mbar_wait(&bars[kFull + slot], (n / kStages) & 1, kErrDecodeFullWait);
        if (alive && j >= 2) alive = mbar_wait(&bars[kSFree + sb], ((j >> 1) + 1) & 1, kErrDecodeFullWait);
        if (!alive) break;
        tc_fence_after();
        const uint32_t k_addr = sbase + kRingOff + slot * kKVBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = sw128_desc(k_addr + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
          const uint64_t b = sw128_desc(q_addr + (kk >> 2) * kNHalf + (kk & 3) * 32, 16, 1024);
          umma(tmem + sb * kN, a, b, kIdescS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&bars[kEmpty + slot]);
        umma_commit(&bars[kSFull + sb]);
        if (j >= 1) issue_pv(j - 1);
      }
      if (alive) issue_pv(ntiles - 1);
    }
  } else {
    // ------------------------------------------------- softmax and epilogue
    const int quad = warp & 3;
    const int t = quad * 32 + lane;  // token of S^T, dimension of O^T
    const uint32_t tlane = tmem + (uint32_t(quad * 32) << 16);
    const float sl2 = p.scale_log2;
    float m_used[kN], lpart[kN];
#pragma unroll
    for (int g = 0; g < kN; ++g) {
      m_used[g] = -INFINITY;
      lpart[g] = 0.0f;
    }
    bool alive = true;
    for (int j = 0; j < ntiles; ++j) {
      const int sb = j & 1;
      const int token0 = (t0 + j) * kTok;
      const int page = table[token0 / p.block_size];
      const bool ok = page >= 0 && page < p.num_blocks;
      if (!mbar_wait(&bars[kSFull + sb], (j >> 1) & 1, kErrDecodeFullWait)) {
        alive = false;
        break;
      }
      tc_fence_after();
      uint32_t raw[16];
      tmem_ld16(tlane + sb * kN, raw);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kSFree + sb]);
      const int tok = token0 + t;
      const bool live = ok && tok < len;
      float x[kN];
#pragma unroll
      for (int g = 0; g < kN; ++g) x[g] = live && g < group ? __uint_as_float(raw[g]) * sl2 : -INFINITY;
      // per-head tile max: warp butterfly, then the 4-warp exchange
      float* ex = exch + (j & 1) * 4 * kN;
#pragma unroll
      for (int g = 0; g < kN; ++g) {
        if (g >= group) break;
        float v = x[g];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if (lane == 0) ex[quad * kN + g] = v;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kXch + (j & 1)]);
      if (!mbar_wait(&bars[kXch + (j & 1)], (j >> 1) & 1, kErrDecodeFullWait)) {
        alive = false;
        break;
      }
      float alpha[kN];
      bool any = false;
#pragma unroll
      for (int g = 0; g < kN; ++g) {
        alpha[g] = 1.0f;
        if (g >= group) continue;
        const float mt = fmaxf(fmaxf(ex[g], ex[kN + g]), fmaxf(ex[2 * kN + g], ex[3 * kN + g]));
        if (mt > m_used[g] + kRescaleLog2) {
          alpha[g] = fast_exp2(m_used[g] - mt);
          m_used[g] = mt;
          any = true;
        }
      }
      float pr[kN];
#pragma unroll
      for (int g = 0; g < kN; ++g) {
        const float me = m_used[g] == -INFINITY ? 0.0f : m_used[g];
        pr[g] = fast_exp2(x[g] - me);  // masked and padded heads give 0
        lpart[g] = lpart[g] * alpha[g] + pr[g];
      }
      // PV_{j-1} must be complete: P^T and, on a rescale, O^T are rewritten.
      if (j >= 1) {
        if (!mbar_wait(&bars[kODone], (j - 1) & 1, kErrDecodeFullWait)) {
          alive = false;
          break;
        }
        tc_fence_after();
      }
      // V rows of tokens that are not real keys are zeroed: P = 0 must never
      // meet a non-finite cache value. The wait is for V_j's load itself:
      // the slot's next load (K_{j+2}) needs PV_j, which needs this P_j.
      if (__any_sync(0xffffffffu, !live)) {
        const int n = 2 * j + 1, slot = n % kStages;
        if (!mbar_wait(&bars[kFull + slot], (n / kStages) & 1, kErrDecodeFullWait)) {
          alive = false;
          break;
        }
        if (!live) {
          const uint32_t vrow = sbase + kRingOff + slot * kKVBytes + t * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            st_shared_zero16(vrow + c * 16);
            st_shared_zero16(vrow + kHalf + c * 16);
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kN; ++g) {
        if (g >= group) break;
        const __nv_bfloat16 hb = __float2bfloat16_rn(pr[g]);
        st_shared_u16(sbase + kPOff + sw_offset(g, t, kNHalf), *reinterpret_cast<const uint16_t*>(&hb));
      }
      fence_proxy_async_smem();
      if (j >= 1 && any) {  // any is uniform: every thread computed the same maxima
        uint32_t o[16];
        tmem_ld16(tlane + kOCol, o);
        tmem_ld_wait();
#pragma unroll
        for (int g = 0; g < kN; ++g) o[g] = __float_as_uint(__uint_as_float(o[g]) * alpha[g]);
        tmem_st16(tlane + kOCol, o);
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kPFull]);
    }

    // epilogue: l = sum of the per-thread partials, then O^T / l
    float* lex = exch;  // reuse as [4][kN]
    named_barrier(1, 128);
#pragma unroll
    for (int g = 0; g < kN; ++g) {
      if (g >= group) break;
      float v = lpart[g];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) lex[quad * kN + g] = v;
    }
    named_barrier(1, 128);
    if (alive && mbar_wait(&bars[kODone], (ntiles - 1) & 1, kErrDecodeFullWait)) {
      tc_fence_after();
      uint32_t o[16];
      tmem_ld16(tlane + kOCol, o);
      tmem_ld_wait();
#pragma unroll
      for (int g = 0; g < kN; ++g) {
        if (g >= group) break;
        const float L = (lex[g] + lex[kN + g]) + (lex[2 * kN + g] + lex[3 * kN + g]);
        const float val = L > 0.0f ? __uint_as_float(o[g]) / L : 0.0f;
        const float m_out = m_used[g] == -INFINITY ? 0.0f : m_used[g];
        const float lse = L > 0.0f ? (m_out + fast_log2(L)) * kLn2 : -INFINITY;
        const long long rh = (long long)row * p.qh + head0 + g;
        if (p.num_splits == 1) {
          p.out[rh * 128 + t] = __float2bfloat16_rn(val);
          if (t == 0 && p.lse) p.lse[lse_base + (long long)(head0 + g) * p.max_q] = lse;
        } else {
          p.out_accum[((long long)split * p.rows * p.qh + rh) * 128 + t] = val;
          if (t == 0) p.lse_accum[(long long)split * p.rows * p.qh + rh] = lse;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace decode_mma_detail

// Returns cudaErrorNotSupported for shapes this kernel does not cover (pages
// that are not a multiple of 128 tokens). p.n_hgroups must be
// ceil(group / 16).
cudaError_t launch_decode_mma(const DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                              const CUtensorMap& kmap_half, const CUtensorMap& vmap_half, cudaStream_t stream) {
  using namespace decode_mma_detail;
  const int group = p.qh / p.kvh;
  if (p.mode != kModeDecode || p.block_size % kTok || p.n_hgroups != (group + kN - 1) / kN)
    return cudaErrorNotSupported;
  static unsigned configured[kContextSlots] = {};
  const cudaError_t e = once_per_context(configured, [] {
    cudaError_t r = cudaFuncSetAttribute(decode_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (r != cudaSuccess) return r;
    return cudaFuncSetAttribute(decode_mma_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared);
  });
  if (e != cudaSuccess) return e;
  const long long grid = (long long)p.rows * p.kvh * p.n_hgroups * p.num_splits;
  if (grid <= 0 || grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  // Programmatic dependent of the kernel before it on the stream: barrier
  // set-up and TMEM allocation overlap that kernel's tail; every global
  // access waits (griddepcontrol.wait) for it to complete.
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_mma_kernel, p, kmap, vmap, kmap_half, vmap_half);
}

}  // namespace nvb
