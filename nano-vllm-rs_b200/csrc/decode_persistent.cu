// Persistent form of the tcgen05 paged decode (decode_mma.cu), for the
// short, ragged contexts of an engine's decode batch: the entry points use it
// when the caller's max_k is at most 2048 tokens (csrc/api.cu).
//
// Same contract, tiles, MMAs and softmax as decode_mma.cu (reference paths:
// kernels/kernels.cu:288-354 and the FA2 decode behind
// kernels/flash_native/flash_native.cu:61-112). The difference is the work
// schedule: one CTA per resident slot (two per SM) claims work items
// (sequence, kv head, 16-head group, split) from a per-stream counter until
// none are left, so an item of a few tiles does not pay a CTA's set-up and
// pipeline ramp: the K/V rings, TMEM and barriers carry over from item to
// item, and the next item's Q^T (by TMA) and first K/V tiles load while the
// current one finishes. Measured on the same B200 with medians of 7
// interleaved rounds: 256 contexts U[128, 1536] at 16q/8kv 0.1562 vs 0.1625
// ms (+4 %); on long contexts (config 3, 4096 tokens; config 5, 32768 in 9
// splits) it was 4-5 % slower than the one-CTA-per-item form, which those
// keep.
//
// Warp roles: warp 0 claims items and streams each item's Q^T and K/V tiles
// (32 KB tiles, K and V sharing one 3-slot ring in the order K0 V0 K1 V1 ...,
// as the one-CTA-per-item kernel does) with 3-D TMA, warp 1 owns TMEM and
// issues the MMAs, warps 2..5 run the softmax and the epilogue. Every
// mbarrier is waited on every phase, in order, by each of its waiters (except
// the softmax's wait for a V tile, taken only on tiles with masked tokens: its
// slot's next load needs this tile's PV, so it cannot run two phases ahead);
// phases count tiles (or items) over the CTA's whole item stream. The softmax warps'
// waits are warp-uniform and bounded, and no role waits at a barrier without
// a time limit.
#include <mutex>

#include "internal.cuh"

namespace nvb {

namespace decode_persistent_detail {

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
// kItemFull / kItemEmpty: the two-slot item ring; kQFull / kQEmpty: the two
// Q^T buffers, used by items in turn; kLex: the epilogue's row-sum exchange.
enum Bar { kFull = 0, kEmpty = kFull + kStages, kSFull = kEmpty + kStages, kSFree = kSFull + 2,
           kPFull = kSFree + 2, kODone = kPFull + 1,
           kXch = kODone + 1, kItemFull = kXch + 2, kItemEmpty = kItemFull + 2, kQFull = kItemEmpty + 2,
           kQEmpty = kQFull + 2, kLex = kQEmpty + 2, kNumBars = kLex + 1 };
constexpr int kTmemSlotOff = kNumBars * 8;
constexpr int kExchOff = kTmemSlotOff + 16;         // float [2][4 warps][16] max exchange
constexpr int kLexOff = kExchOff + 2 * 4 * kN * 4;  // float [4 warps][16] row sums
constexpr int kRingOff = kLexOff + 4 * kN * 4;      // Item [2]
constexpr int kHeadBytes = kRingOff + 2 * 28;  // sizeof(Item) == 28, checked below
static_assert(kHeadBytes <= 1024, "barrier block must fit below the first 1 KB boundary");
// Tile load n (K of the CTA's tile n / 2 when n is even, its V when odd)
// uses slot n % kStages.
constexpr int kSlotOff = 0;
constexpr int kQOff = kSlotOff + kStages * kKVBytes;
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

// One work item: the keys [t0, t0 + ntiles) tiles of one (sequence, kv head,
// 16-head group, split). row < 0 ends the CTA's item stream.
struct Item {
  int row, kvhead, hgroup, split, t0, ntiles, len;
};

static_assert(sizeof(Item) == 28, "the item ring holds two 28-byte entries");

__device__ __forceinline__ Item make_item(const DecodeParams& p, int v) {
  Item it;
  it.split = v % p.num_splits;
  v /= p.num_splits;
  it.hgroup = v % p.n_hgroups;
  v /= p.n_hgroups;
  it.kvhead = v % p.kvh;
  it.row = v / p.kvh;
  it.len = p.lens[it.row];
  const bool valid = it.len >= 1 && (long long)it.len <= (long long)p.table_stride * p.block_size;
  const int total = valid ? (it.len + kTok - 1) / kTok : 0;
  const int per_split = (total + p.num_splits - 1) / p.num_splits;
  it.t0 = it.split * per_split;
  it.ntiles = max(0, min(it.t0 + per_split, total) - it.t0);
  return it;
}

__global__ void __launch_bounds__(kThreads, 2)
    decode_persistent_kernel(const DecodeParams p, int* sched, const __grid_constant__ CUtensorMap kmap,
                             const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap kmap_half,
                             const __grid_constant__ CUtensorMap vmap_half, const __grid_constant__ CUtensorMap qmap) {
  // The kernel after this grid on the stream, when launched with
  // programmatic stream serialization (a split-KV combine), may be scheduled
  // now; it waits (griddepcontrol.wait) for this grid to complete before it
  // reads the partials.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  const uint32_t tile_addr = (raw_addr + kHeadBytes + 1023u) & ~1023u;
  unsigned char* tiles = smem_raw + (tile_addr - raw_addr);
  const uint32_t sbase = tile_addr;
  if (tile_addr + kTileBytes > raw_addr + kSmemBytes) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (threadIdx.x == 0) record_error(kErrPrefillAlign);
    return;
  }
  const int group_total = p.qh / p.kvh;
  const int n_items = p.rows * p.kvh * p.n_hgroups * p.num_splits;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_raw + kTmemSlotOff);
  float* exch = reinterpret_cast<float*>(smem_raw + kExchOff);  // [2][4][kN]
  float* lex = reinterpret_cast<float*>(smem_raw + kLexOff);    // [4][kN]
  Item* ring = reinterpret_cast<Item*>(smem_raw + kRingOff);    // [2]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kFull + s], 1);
      mbar_init(&bars[kEmpty + s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kSFull + s], 1);
      mbar_init(&bars[kSFree + s], 4);
      mbar_init(&bars[kXch + s], 4);
      mbar_init(&bars[kItemFull + s], 1);
      mbar_init(&bars[kItemEmpty + s], 5);  // the MMA thread + the 4 softmax warps
      mbar_init(&bars[kQFull + s], 1);
      mbar_init(&bars[kQEmpty + s], 1);
    }
    mbar_init(&bars[kPFull], 4);
    mbar_init(&bars[kODone], 1);
    mbar_init(&bars[kLex], 4);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp >= 2) {
    // Rows >= group of P^T start at zero. (A later item with a smaller head
    // group leaves stale rows past its group: they only reach O^T columns
    // that its epilogue never reads, and S^T columns past the group are
    // masked.)
    const int t = threadIdx.x - 64;
    for (int e = t; e < kN * 16; e += 128) {
      const int g = e >> 4, chunk = e & 15;
      if (g >= group_total) st_shared_zero16(sbase + kPOff + sw_offset(g, chunk * 8, kNHalf));
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Launched as a programmatic dependent of the previous kernel on the
  // stream: the set-up above touches only this CTA's shared memory and TMEM
  // and overlaps that kernel's tail. Wait for it to complete, its writes
  // (the new tokens' K/V and queries, this stream's claim-counter reset)
  // visible, before any global access.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    // ------------------------------------------ item claims and producer
    // Claims items from the stream's counter one at a time (each claim comes
    // when the previous item's loads are issued, so the last claims balance
    // the CTAs), publishes them in a two-slot ring, loads each item's Q^T
    // [16 heads][128 dims] (heads past the group are other heads or zero
    // fill, whose scores the softmax ignores) and streams its K/V tiles. Ring
    // stages and barrier phases count tiles over the CTA's whole item stream.
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      tma_prefetch_desc(&kmap_half);
      tma_prefetch_desc(&vmap_half);
      tma_prefetch_desc(&qmap);
      const uint64_t policy = policy_evict_first();
      int g = 0, ni = 0;
      // The first item is the CTA's own index; later claims count on from
      // gridDim.x, so the launch does not start with every CTA's atomic on
      // one address.
      int v = blockIdx.x;
      for (int i = 0;; ++i) {
        Item it;
        if (v < n_items) {
          it = make_item(p, v);
        } else {
          it.row = -1;
          it.ntiles = 0;
        }
        if (i >= 2 && !mbar_wait(&bars[kItemEmpty + (i & 1)], ((i >> 1) + 1) & 1, kErrDecodeEmptyWait)) break;
        ring[i & 1] = it;
        mbar_arrive(&bars[kItemFull + (i & 1)]);
        if (it.row < 0) break;
        if (it.ntiles == 0) {
          v = int(gridDim.x) + atomicAdd(sched, 1);
          continue;
        }
        const int qb = ni & 1;
        if (ni >= 1 && !mbar_wait(&bars[kQEmpty], ((ni - 1) & 1), kErrDecodeEmptyWait)) break;
        mbar_arrive_expect_tx(&bars[kQFull + qb], kNBytes);
        const uint32_t qd = sbase + kQOff;
        const int qhead0 = it.kvhead * group_total + it.hgroup * kN;
        tma_load_3d_plain(qd, &qmap, &bars[kQFull + qb], 0, qhead0, it.row);
        tma_load_3d_plain(qd + kNHalf, &qmap, &bars[kQFull + qb], 64, qhead0, it.row);
        ++ni;
        const int* table = p.block_table + (long long)it.row * p.table_stride;
        bool alive = true;
        const int claim_at = it.ntiles > 2 ? it.ntiles - 2 : 0;
        for (int j = 0; j < it.ntiles; ++j, ++g) {
          if (j == claim_at) v = int(gridDim.x) + atomicAdd(sched, 1);
          const int token0 = (it.t0 + j) * kTok;
          const int logical = token0 / p.block_size;
          const int page = table[logical];
          const bool ok = page >= 0 && page < p.num_blocks;
          const int trow = ok ? page * p.block_size + (token0 - logical * p.block_size) : 0;
          // A sequence's last tile with at most 64 live tokens loads 64 rows.
          const bool half = it.len - token0 <= kTok / 2;
          const uint32_t tile_bytes = half ? kKVBytes / 2 : kKVBytes;
          // K then V of the tile; each slot's previous load (n - kStages) is
          // released by the MMA that read it (S of a K tile, PV of a V tile).
          for (int n = 2 * g; n <= 2 * g + 1; ++n) {
            const CUtensorMap* m = (n & 1) ? (half ? &vmap_half : &vmap) : (half ? &kmap_half : &kmap);
            const int slot = n % kStages;
            if (n >= kStages && !mbar_wait(&bars[kEmpty + slot], ((n / kStages) + 1) & 1, kErrDecodeEmptyWait)) {
              alive = false;
              break;
            }
            if (ok) {
              unsigned char* d = tiles + kSlotOff + slot * kKVBytes;
              mbar_arrive_expect_tx(&bars[kFull + slot], tile_bytes);
              tma_load_3d_hint(d, m, &bars[kFull + slot], 0, it.kvhead, trow, policy);
              tma_load_3d_hint(d + kHalf, m, &bars[kFull + slot], 64, it.kvhead, trow, policy);
            } else {
              mbar_arrive(&bars[kFull + slot]);
            }
          }
          if (!alive) break;
        }
        if (!alive) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool alive = true;
      const uint32_t p_addr = sbase + kPOff;
      // PV of global tile g; `first` starts the item's accumulator.
      auto issue_pv = [&](int g, bool first) {
        const int n = 2 * g + 1, slot = n % kStages;
        alive = alive && mbar_wait(&bars[kPFull], g & 1, kErrDecodeFullWait);
        alive = alive && mbar_wait(&bars[kFull + slot], (n / kStages) & 1, kErrDecodeFullWait);
        if (!alive) return;
        tc_fence_after();
        const uint32_t v_addr = sbase + kSlotOff + slot * kKVBytes;
#pragma unroll
        for (int kk = 0; kk < kTok / 16; ++kk) {
          // A = V^T, MN-major: 64-dim halves kHalf apart, 8-token groups 1 KB apart
          const uint64_t a = sw128_desc(v_addr + kk * 2048, kHalf, 1024);
          const uint64_t b = sw128_desc(p_addr + (kk >> 2) * kNHalf + (kk & 3) * 32, 16, 1024);
          umma(tmem + kOCol, a, b, kIdescPV, (!first || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars[kEmpty + slot]);
        umma_commit(&bars[kODone]);
      };
      int g = 0, ni = 0;
      for (int i = 0; alive; ++i) {
        if (!mbar_wait(&bars[kItemFull + (i & 1)], (i >> 1) & 1, kErrDecodeFullWait)) break;
        const Item it = ring[i & 1];
        mbar_arrive(&bars[kItemEmpty + (i & 1)]);
        if (it.row < 0) break;
        if (it.ntiles == 0) continue;
        const int qb = ni & 1;
        if (!mbar_wait(&bars[kQFull + qb], (ni >> 1) & 1, kErrDecodeFullWait)) break;
        ++ni;
        const uint32_t q_addr = sbase + kQOff;
        for (int j = 0; j < it.ntiles && alive; ++j, ++g) {
          const int n = 2 * g, slot = n % kStages, sb = g & 1;
          alive = mbar_wait(&bars[kFull + slot], (n / kStages) & 1, kErrDecodeFullWait);
          if (alive && g >= 2) alive = mbar_wait(&bars[kSFree + sb], ((g >> 1) + 1) & 1, kErrDecodeFullWait);
          if (!alive) break;
          tc_fence_after();
          const uint32_t k_addr = sbase + kSlotOff + slot * kKVBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t a = sw128_desc(k_addr + (kk >> 2) * kHalf + (kk & 3) * 32, 16, 1024);
            const uint64_t b = sw128_desc(q_addr + (kk >> 2) * kNHalf + (kk & 3) * 32, 16, 1024);
            umma(tmem + sb * kN, a, b, kIdescS, kk > 0 ? 1u : 0u);
          }
          umma_commit(&bars[kEmpty + slot]);
          umma_commit(&bars[kSFull + sb]);
          if (j == it.ntiles - 1) umma_commit(&bars[kQEmpty]);
          if (j >= 1) issue_pv(g - 1, j == 1);
        }
        // The item's last PV goes out before the next item's first S, so the
        // epilogue's wait for it never depends on the next item's loads.
        if (alive) issue_pv(g - 1, it.ntiles == 1);
      }
    }
  } else {
    // ------------------------------------------------- softmax and epilogue
    const int quad = warp & 3;
    const int t = quad * 32 + lane;  // token of S^T, dimension of O^T
    const uint32_t tlane = tmem + (uint32_t(quad * 32) << 16);
    const float sl2 = p.scale_log2;
    // Every wait here is warp-uniform (a lane that gives up makes the whole
    // warp give up), and no wait is unbounded: a failure anywhere ends the
    // warp's loop without leaving another warp at a barrier it cannot pass.
    auto wwait = [](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, kErrDecodeFullWait));
    };
    bool alive = true;
    int g = 0, ni = 0;
    for (int i = 0; alive; ++i) {
      if (!wwait(&bars[kItemFull + (i & 1)], (i >> 1) & 1)) break;
      const Item it = ring[i & 1];
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kItemEmpty + (i & 1)]);
      if (it.row < 0) break;
      const int head0 = it.kvhead * group_total + it.hgroup * kN;
      const int group = min(kN, group_total - it.hgroup * kN);  // this item's heads
      if (it.ntiles == 0) {
        for (int gg = 0; gg < group; ++gg) {
          const long long rh = (long long)it.row * p.qh + head0 + gg;
          if (p.num_splits == 1) {
            p.out[rh * 128 + t] = __float2bfloat16_rn(0.0f);
            if (t == 0 && p.lse) p.lse[(long long)it.row * p.qh * p.max_q + (long long)(head0 + gg) * p.max_q] =
                -INFINITY;
          } else {
            p.out_accum[((long long)it.split * p.rows * p.qh + rh) * 128 + t] = 0.0f;
            if (t == 0) p.lse_accum[(long long)it.split * p.rows * p.qh + rh] = -INFINITY;
          }
        }
        continue;
      }
      const int* table = p.block_table + (long long)it.row * p.table_stride;
      float m_used[kN], lpart[kN];
#pragma unroll
      for (int gg = 0; gg < kN; ++gg) {
        m_used[gg] = -INFINITY;
        lpart[gg] = 0.0f;
      }
      for (int j = 0; j < it.ntiles; ++j, ++g) {
        const int sb = g & 1;
        const int token0 = (it.t0 + j) * kTok;
        const int page = table[token0 / p.block_size];
        const bool ok = page >= 0 && page < p.num_blocks;
        if (!wwait(&bars[kSFull + sb], (g >> 1) & 1)) {
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
        const bool live = ok && tok < it.len;
        float x[kN];
#pragma unroll
        for (int gg = 0; gg < kN; ++gg) x[gg] = live && gg < group ? __uint_as_float(raw[gg]) * sl2 : -INFINITY;
        // per-head tile max: warp butterfly, then the 4-warp exchange
        float* ex = exch + (g & 1) * 4 * kN;
#pragma unroll
        for (int gg = 0; gg < kN; ++gg) {
          if (gg >= group) break;
          float v = x[gg];
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
          if (lane == 0) ex[quad * kN + gg] = v;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kXch + (g & 1)]);
        if (!wwait(&bars[kXch + (g & 1)], (g >> 1) & 1)) {
          alive = false;
          break;
        }
        float alpha[kN];
        bool any = false;
#pragma unroll
        for (int gg = 0; gg < kN; ++gg) {
          alpha[gg] = 1.0f;
          if (gg >= group) continue;
          const float mt = fmaxf(fmaxf(ex[gg], ex[kN + gg]), fmaxf(ex[2 * kN + gg], ex[3 * kN + gg]));
          if (mt > m_used[gg] + kRescaleLog2) {
            alpha[gg] = fast_exp2(m_used[gg] - mt);
            m_used[gg] = mt;
            any = true;
          }
        }
        float pr[kN];
#pragma unroll
        for (int gg = 0; gg < kN; ++gg) {
          const float me = m_used[gg] == -INFINITY ? 0.0f : m_used[gg];
          pr[gg] = fast_exp2(x[gg] - me);  // masked and padded heads give 0
          lpart[gg] = lpart[gg] * alpha[gg] + pr[gg];
        }
        // PV of the previous tile must be complete: P^T and, on a rescale,
        // O^T are rewritten. (An item's first tile follows its predecessor's
        // epilogue, which already waited for that item's last PV.)
        if (j >= 1) {
          if (!wwait(&bars[kODone], (g - 1) & 1)) {
            alive = false;
            break;
          }
          tc_fence_after();
        }
        // V rows of tokens that are not real keys are zeroed: P = 0 must
        // never meet a non-finite cache value. The wait is for V of tile g
        // itself: the slot's next load (K of tile g + 2) needs PV of tile g,
        // which needs this P.
        if (__any_sync(0xffffffffu, !live)) {
          const int n = 2 * g + 1, slot = n % kStages;
          if (!wwait(&bars[kFull + slot], (n / kStages) & 1)) {
            alive = false;
            break;
          }
          if (!live) {
            const uint32_t vrow = sbase + kSlotOff + slot * kKVBytes + t * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              st_shared_zero16(vrow + c * 16);
              st_shared_zero16(vrow + kHalf + c * 16);
            }
          }
        }
#pragma unroll
        for (int gg = 0; gg < kN; ++gg) {
          if (gg >= group) break;
          const __nv_bfloat16 hb = __float2bfloat16_rn(pr[gg]);
          st_shared_u16(sbase + kPOff + sw_offset(gg, t, kNHalf), *reinterpret_cast<const uint16_t*>(&hb));
        }
        fence_proxy_async_smem();
        if (j >= 1 && any) {  // any is uniform: every thread computed the same maxima
          uint32_t o[16];
          tmem_ld16(tlane + kOCol, o);
          tmem_ld_wait();
#pragma unroll
          for (int gg = 0; gg < kN; ++gg) o[gg] = __float_as_uint(__uint_as_float(o[gg]) * alpha[gg]);
          tmem_st16(tlane + kOCol, o);
          tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kPFull]);
      }
      if (!alive) break;

      // epilogue: l = sum of the per-thread partials, then O^T / l. The
      // four warps' sums meet through kLex (one phase per item). lex is
      // rewritten by the next item's epilogue only after every warp has
      // passed that item's first max exchange, i.e. finished reading it here.
#pragma unroll
      for (int gg = 0; gg < kN; ++gg) {
        if (gg >= group) break;
        float v = lpart[gg];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) lex[quad * kN + gg] = v;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kLex]);
      if (!wwait(&bars[kLex], ni & 1)) break;
      ++ni;
      if (!wwait(&bars[kODone], (g - 1) & 1)) break;
      tc_fence_after();
      uint32_t o[16];
      tmem_ld16(tlane + kOCol, o);
      tmem_ld_wait();
      tc_fence_before();
      const long long lse_base = (long long)it.row * p.qh * p.max_q;
#pragma unroll
      for (int gg = 0; gg < kN; ++gg) {
        if (gg >= group) break;
        const float L = (lex[gg] + lex[kN + gg]) + (lex[2 * kN + gg] + lex[3 * kN + gg]);
        const float val = L > 0.0f ? __uint_as_float(o[gg]) / L : 0.0f;
        const float m_out = m_used[gg] == -INFINITY ? 0.0f : m_used[gg];
        const float lse = L > 0.0f ? (m_out + fast_log2(L)) * kLn2 : -INFINITY;
        const long long rh = (long long)it.row * p.qh + head0 + gg;
        if (p.num_splits == 1) {
          p.out[rh * 128 + t] = __float2bfloat16_rn(val);
          if (t == 0 && p.lse) p.lse[lse_base + (long long)(head0 + gg) * p.max_q] = lse;
        } else {
          p.out_accum[((long long)it.split * p.rows * p.qh + rh) * 128 + t] = val;
          if (t == 0) p.lse_accum[(long long)it.split * p.rows * p.qh + rh] = lse;
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
  if (threadIdx.x == 0) {
    // The last CTA to finish resets the claim counter for the next launch on
    // this stream (every CTA's claims precede its increment here).
    __threadfence();
    if (atomicAdd(sched + 1, 1) == int(gridDim.x) - 1) {
      atomicExch(sched, 0);
      atomicExch(sched + 1, 0);
    }
  }
}

// Claim counters {next item, CTAs finished}, one pair per stream that
// launches the decode (a launch leaves its pair at zero when it ends).
__device__ int g_persistent_sched[64][2];

// Pair for (stream, context): streams get their own pair in order of first
// use; past 64 streams pairs are shared by hash, and launches sharing a pair
// must not overlap in time. A captured graph keeps the pair of the stream it
// was captured on.
int* sched_pair(cudaStream_t stream, cudaError_t* err) {
  static std::mutex mu;
  static int* base[kContextSlots] = {};
  static unsigned base_gen[kContextSlots] = {};
  static cudaStream_t keys[kContextSlots][64];
  static int used[kContextSlots] = {};
  int ctx = 0;
  unsigned gen = 0;
  if (int rc = context_slot(&ctx, &gen)) {
    *err = cudaError_t(rc);
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (base_gen[ctx] != gen) {
    void* ptr = nullptr;
    *err = cudaGetSymbolAddress(&ptr, g_persistent_sched);
    if (*err != cudaSuccess) return nullptr;
    base[ctx] = static_cast<int*>(ptr);
    base_gen[ctx] = gen;
    used[ctx] = 0;
  }
  int slot = -1;
  for (int i = 0; i < used[ctx]; ++i)
    if (keys[ctx][i] == stream) slot = i;
  if (slot < 0 && used[ctx] < 64) {
    keys[ctx][used[ctx]] = stream;
    slot = used[ctx]++;
  }
  if (slot < 0) slot = int((reinterpret_cast<uintptr_t>(stream) >> 4) & 63);
  return base[ctx] + 2 * slot;
}

}  // namespace decode_persistent_detail

// Returns cudaErrorNotSupported for shapes this kernel does not cover (pages
// that are not a multiple of 128 tokens). p.n_hgroups must be
// ceil(group / 16).
cudaError_t launch_decode_persistent(const DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                                     const CUtensorMap& kmap_half, const CUtensorMap& vmap_half,
                                     const CUtensorMap& qmap, cudaStream_t stream) {
  using namespace decode_persistent_detail;
  const int group = p.qh / p.kvh;
  if (p.mode != kModeDecode || p.block_size % kTok || p.n_hgroups != (group + kN - 1) / kN)
    return cudaErrorNotSupported;
  static unsigned configured[kContextSlots] = {};
  static int resident[kContextSlots] = {};
  int slot = 0;
  unsigned gen = 0;
  if (int rc = context_slot(&slot, &gen)) return cudaError_t(rc);
  const cudaError_t e = once_per_context(configured, [slot] {
    cudaError_t r =
        cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (r != cudaSuccess) return r;
    r = cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (r != cudaSuccess) return r;
    int dev = 0, sms = 0;
    if ((r = cudaGetDevice(&dev)) != cudaSuccess) return r;
    if ((r = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return r;
    // Two CTAs per SM (the launch bounds and the shared-memory budget are set
    // for it). A CTA that finds no slot only starts late and finds the items
    // claimed.
    __atomic_store_n(&resident[slot], 2 * sms, __ATOMIC_RELEASE);
    return cudaSuccess;
  });
  if (e != cudaSuccess) return e;
  cudaError_t se = cudaSuccess;
  int* sched = sched_pair(stream, &se);
  if (!sched) return se == cudaSuccess ? cudaErrorUnknown : se;
  const long long items = (long long)p.rows * p.kvh * p.n_hgroups * p.num_splits;
  if (items <= 0 || items > 0x7fffffffLL) return cudaErrorInvalidValue;
  const int slots = __atomic_load_n(&resident[slot], __ATOMIC_ACQUIRE);
  const unsigned grid = unsigned(items < slots ? items : slots);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_persistent_kernel, p, sched, kmap, vmap, kmap_half, vmap_half, qmap);
}

}  // namespace nvb
