// Varlen / chunked causal prefill over the paged KV cache on tcgen05 tensor
// cores (sm_100a).
//
// Replaces the reference's prefill paths: FA2's paged split-KV kernel with
// num_splits = 1 and a bottom-right causal mask (SM80 mma.sync, launched from
// kernels/flash_native/flash_native.cu:102-112) and the native ordered kernel
// (kernels/kernels.cu:288-354, one CTA per query row). The causal rule is the
// reference's: query i of a q_len-query group sees keys
// [0, kv_len - q_len + i] (src/model.rs:1170-1188, smoke.cu:58).
//
// Work item: a pair of adjacent 128-row query tiles A and B of one (sequence,
// kv head). Rows pack the GQA group: row r of a tile is (query q0 + r / G,
// head h*G + r % G), so each K/V tile serves every query head of the group,
// and both tiles of the pair. Per 128-key KV tile j and tile x in {A, B}:
//
//   S_x = Q_x K_j^T   tcgen05.mma kind::f16, M=128 N=128 K=128 (8 x K16), A and
//                     B from 128B-swizzled shared memory, D in TMEM (FP32)
//   P_x = exp2(S_x * scale*log2e - m)   softmax warpgroup x, each thread one
//                     row and all 128 keys; P written back over S_x in TMEM as
//                     packed BF16
//   O_x += P_x V_j    tcgen05.mma M=128 N=128 K=128, A (P) read from TMEM, V an
//                     MN-major B operand in shared memory, O_x in TMEM
//
// TMEM: S_A 0, S_B 128, O_A 256, O_B 384 (512 columns). S_x is single-buffered,
// so each tile's chain is softmax -> PV -> next S -> softmax; the two tiles'
// chains run out of phase on the tensor core (S_A, S_B, PV_A, PV_B), so one
// softmax warpgroup's loads and max overlap the other's exponentials, and no
// thread exchanges a row max with another. Sequences whose queries all fit
// one tile (short chunks) go to the one-tile kernel in prefill_tile.cu, where
// a pair would leave tile B empty.
//
// Roles (16 warps, one CTA per SM):
//   warp 0      claims items (global counter, heaviest first), publishes each
//               to the CTA through a two-slot ring, loads Q_A and Q_B (one
//               buffer each, reloaded when the tile's last S has read it) and
//               the K tiles (two-stage ring) with TMA: 3-D maps over [tokens,
//               kv_heads, 128], 64-element 128-byte-swizzled boxes; a 128-key
//               tile never crosses a page since block_size is a multiple of 256
//   warp 1      TMEM owner; one thread issues the S MMAs and their commits
//   warp 2      V fixer and PV issuer: zeroes V rows that are not real keys
//               (past kv_len or an invalid page) so P ~ 0 never meets a
//               non-finite cache value, then one thread issues the tile's PV
//               MMAs once P is in TMEM (two issuing threads: neither the S
//               nor the PV stream waits behind the other's barriers)
//   warp 3      loads the V tiles (two-stage ring)
//   warps 4-7   softmax of tile A; warps 8-11 softmax of tile B (200 registers
//               a thread through setmaxnreg: a row's 128 scores stay in
//               registers)
//   warps 12-15 epilogue: O_x / l -> BF16 rows and the LSE, from row statistics
//               handed over in shared memory; frees O_x for its next tile
//
// The softmax keeps the running max it scales by unless a row's max grows by
// more than 2^8 (lazy rescale: P stays <= 256, exact after the final divide),
// so the TMEM read-modify-write of O is rare. An eighth of the exponentials
// run on the FMA pipe (exp2_fma_pair).
//
// mbarrier parity waits are sound only if a waiter is never two phases
// behind or ahead of the barrier; every barrier below is waited at every
// phase, in order, by each role that waits on it, and its next phase needs
// that role's progress. Every wait is bounded (common.cuh); a timeout records
// an error code, the CTA drains its in-flight copies and MMAs (bounded), frees
// TMEM and exits.
#include <mutex>

#include "prefill_common.cuh"

namespace nvb {

namespace prefill_detail {

using namespace prefill_common;

constexpr int kRows = 128;                   // query rows per Q tile (TMEM lanes)
constexpr int kKeys = 128;                   // keys per KV tile
constexpr int kHalf = 128 * 128;             // 128 rows x 64 BF16 (one 128-byte swizzle column)
constexpr int kQBytes = 2 * kHalf;           // Q tile 128 x 128 BF16
constexpr int kKVBytes = 2 * kHalf;          // K or V tile 128 x 128 BF16
constexpr int kQStages = 2, kKStages = 2, kVStages = 2;  // Q: tiles A and B of the item
constexpr int kThreads = 512;
constexpr int kTmemCols = 512;
constexpr int kSCol = 0, kOCol = 256;        // S/P of tile x at kSCol + 128 x, O at kOCol + 128 x
constexpr float kLn2 = 0.693147180559945309f;
constexpr float kRescaleLog2 = 8.0f;         // lazy rescale threshold (P <= 2^8)
// Register split after set-up (launch: 512 threads x 128 a thread): the two
// softmax warpgroups hold a tile row's 128 scores; the producer/MMA and
// epilogue warpgroups run on the rest.
constexpr int kLaunchRegs = 128, kSoftmaxRegs = 200, kOtherRegs = 56;
static_assert(2 * 128 * kSoftmaxRegs + 2 * 128 * kOtherRegs == kThreads * kLaunchRegs, "register split");

// mbarriers, [2] = per Q tile (A, B) or per ring stage
enum Bar {
  kQFull = 0, kQFree = 2, kKFull = 4, kKEmpty = 6, kVFull = 8, kVEmpty = 10,
  kSFull = 12, kPFull = 14, kPVDone = 16, kODone = 18, kOFree = 20, kStatsFull = 22, kStatsFree = 24,
  kItemFull = 26, kItemEmpty = 28,
  kDrain = 30, kPVDrain = 31, kNumBars = 32
};
// Readers of each published item: V producer, S issuer, V fixer (one
// arrival each) and the 8 softmax + 4 epilogue warps (one per warp).
constexpr int kItemReaders = 15;
constexpr int kTmemSlotOff = kNumBars * 8;
constexpr int kItemOff = 320;                               // Item [2] (the published-item ring)
constexpr int kItemBytes = 64;
constexpr int kVRealOff = 448;                              // int [2]: real keys of the V tile in each stage
constexpr int kStatsOff = 512;                              // float2 [2][128]: row max used, row sum
constexpr int kMaxSorted = 1024;                            // batches up to this size are claimed by work
constexpr int kOrderOff = kStatsOff + 2 * kRows * 8;        // int [kMaxSorted]: sequences, heaviest first
constexpr int kWorkOff = kOrderOff + kMaxSorted * 4;        // float [kMaxSorted]: each sequence's work
constexpr int kHeadBytes = kWorkOff + kMaxSorted * 4;
constexpr int kQOff = 0;                                    // offsets from the 1 KB aligned tile base
constexpr int kKOff = kQOff + kQStages * kQBytes;
constexpr int kVOff = kKOff + kKStages * kKVBytes;
constexpr int kTileBytes = kVOff + kVStages * kKVBytes;     // 192 KB
constexpr int kSmemBytes = kTileBytes + kHeadBytes + 1024;  // + worst-case alignment pad
static_assert(kTmemSlotOff + 4 <= kItemOff && kItemOff + 2 * kItemBytes <= kVRealOff && kVRealOff + 8 <= kStatsOff,
              "head layout overlaps");
static_assert(kSmemBytes <= 232448, "tile layout exceeds the per-CTA shared memory limit");

struct PrefillParams {
  int n_qtiles;  // query tiles of the longest sequence
  const int* cu_q;
  const int* kv_lens;
  const int* block_table;
  __nv_bfloat16* out;
  float* lse;
  int batch, max_q, qh, kvh, group, qt, rows_used, block_size, table_stride, num_blocks;
  float scale_log2;
  int* sched;  // {next item to claim, CTAs finished}: zero at launch, reset by the last CTA
  int n_pairs;  // query-tile pairs of the longest sequence
  FastDiv fd_npair, fd_kvh, fd_qt, fd_bs;  // by n_pairs, kvh, qt, block_size
};

// Two adjacent 128-row query tiles (A = q-tile 2k, B = q-tile 2k + 1) of one
// (sequence, kv head): the work item of the persistent loop. A and B share
// every K/V tile; each has its own S/P and O in TMEM and its own softmax
// warpgroup. Virtual items are grouped by (sequence, kv head), longest pair
// first within a group, so the CTAs running at one time share a few groups'
// K/V in L2; the sequences come heaviest first (ranked at kernel start for
// batches up to kMaxSorted) and CTAs claim items from a global counter
// (dynamic load balancing), so the last claims are small ones.
struct Item {
  int b, h, q_begin, kv_len, prefix;
  int q0[2];       // first query of tile A / B within the sequence
  int qx[2];       // queries in the tile (0: tile B is past the sequence)
  int n[2];        // KV tiles the tile visits (0 for an empty tile)
  int full[2];     // leading KV tiles every row of the tile sees whole
  int key_end[2];  // keys the tile's last query sees
};
static_assert(sizeof(Item) <= kItemBytes, "item ring slot too small");

__device__ __forceinline__ int item_tiles(const Item& it) { return max(it.n[0], it.n[1]); }

// `order` (or null): sequence of each rank, heaviest first.
__device__ __forceinline__ Item make_item(const PrefillParams& p, const int* order, int v) {
  Item it;
  const int group = p.fd_npair.div(v);
  const int pair = p.n_pairs - 1 - (v - group * p.n_pairs);
  const int rank = p.fd_kvh.div(group);
  it.b = order ? order[rank] : rank;
  it.h = group - rank * p.kvh;
  it.q_begin = p.cu_q[it.b];
  const int q_len = p.cu_q[it.b + 1] - it.q_begin;
  it.kv_len = p.kv_lens[it.b];
  it.prefix = it.kv_len - q_len;
  // A context longer than the page table, or shorter than its query group,
  // is invalid input: such rows get zero output (as decode does).
  const bool ctx_ok = it.prefix >= 0 && (long long)it.kv_len <= (long long)p.table_stride * p.block_size;
#pragma unroll
  for (int x = 0; x < 2; ++x) {
    it.q0[x] = (2 * pair + x) * p.qt;
    it.qx[x] = max(0, min(p.qt, q_len - it.q0[x]));
    const bool ok = ctx_ok && it.qx[x] > 0;
    it.key_end[x] = ok ? min(it.kv_len, it.prefix + it.q0[x] + it.qx[x]) : 0;
    it.n[x] = (it.key_end[x] + kKeys - 1) / kKeys;
    it.full[x] = ok ? min(it.kv_len, it.prefix + it.q0[x] + 1) / kKeys : 0;
  }
  return it;
}

// Item i of this CTA from the two-slot ring the scheduler publishes.
// `warp_level`: every lane reads it and lane 0 arrives for the warp.
// Returns false at the end marker (b < 0) or if the wait gave up.
__device__ __forceinline__ bool take_item(uint64_t* bars, const Item* ring, int i, bool warp_level, Item& it) {
  const int slot = i & 1;
  const uint32_t par = (i >> 1) & 1;
  if (warp_level) {
    if (!warp_wait(&bars[kItemFull + slot], par)) return false;
  } else if (!mbar_wait(&bars[kItemFull + slot], par, kErrPrefillWait)) {
    return false;
  }
  it = ring[slot];
  if (warp_level) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&bars[kItemEmpty + slot]);
  } else {
    mbar_arrive(&bars[kItemEmpty + slot]);
  }
  return it.b >= 0;
}

// exp2(s * sl2 + nm) for keys [C0, C0 + 32) of a row -> 16 packed BF16 pairs;
// row-sum partials accumulate in `sum`. One pair in eight runs on the FMA pipe.
template <int C0>
__device__ __forceinline__ void exp32(const float (&s)[128], float sl2, float nm, uint32_t (&pk)[16],
                                      float (&sum)[8]) {
#pragma unroll
  for (int c = C0; c < C0 + 32; c += 2) {
    float e0 = s[c], e1 = s[c + 1];
    fma2(e0, e1, e0, e1, sl2, sl2, nm, nm);
    if ((c & 15) == 14) {
      exp2_fma_pair(e0, e1);
    } else {
      e0 = fast_exp2(e0);
      e1 = fast_exp2(e1);
    }
    const int k = (c >> 1) & 3;  // four independent accumulator pairs
    add2(sum[2 * k], sum[2 * k + 1], sum[2 * k], sum[2 * k + 1], e0, e1);
    pk[(c - C0) >> 1] = pack_bf16x2(e0, e1);
  }
}

// Softmax of Q tile x (warps 4-7: A, 8-11: B): one thread per row, all 128
// keys of each KV tile, so no other thread takes part in a row's max. P goes
// back over the first 64 columns of S_x as packed BF16. The running max only
// moves when a row's max grows by more than 2^8 (lazy rescale); O_x is then
// rescaled here, and is quiescent: S_x of this tile was issued after PV_x of
// the previous one completed, and PV_x of this tile waits for this P.
__device__ __forceinline__ void softmax_role(const PrefillParams& p, uint64_t* bars, const Item* ring, float2* stats,
                                             uint32_t tmem, int warp, int lane) {
  const int x = (warp - 4) >> 2;
  const int quad = warp & 3;
  const int r = quad * 32 + lane;  // TMEM lane = packed row
  const uint32_t lane_base = tmem + (uint32_t(quad * 32) << 16);
  const uint32_t scol = lane_base + kSCol + x * kKeys, ocol = lane_base + kOCol + x * kKeys;
  const int rq = r / p.group;
  const float sl2 = p.scale_log2;
  int t = 0, ix = 0;  // tiles and items of this Q tile
  bool alive = true;
  Item it;
  for (int i = 0; alive && take_item(bars, ring, i, true, it); ++i) {
    // this tile's fields (selects: a run-time index would put the item in local memory)
    const int n = x ? it.n[1] : it.n[0];
    if (n == 0) continue;
    const int full = x ? it.full[1] : it.full[0];
    const int qx = x ? it.qx[1] : it.qx[0], q0 = x ? it.q0[1] : it.q0[0];
    const int key_end = x ? it.key_end[1] : it.key_end[0];
    const int* table = p.block_table + (long long)it.b * p.table_stride;
    const bool valid_row = r < p.rows_used && rq < qx;
    const int limit = valid_row ? it.prefix + q0 + rq : key_end - 1;  // last visible key
    float m_used = -INFINITY, l = 0.0f;  // running max the probabilities are scaled by
    for (int j = 0; j < n; ++j, ++t) {
      const int key0 = j * kKeys;
      const bool ok = page_ok(table[p.fd_bs.div(key0)], p.num_blocks);
      if (!warp_wait(&bars[kSFull + x], t & 1)) {
        alive = false;
        break;
      }
      tc_fence_after();
      float s[128];
      {
        uint32_t a0[32], a1[32], a2[32], a3[32];
        tmem_ld32(scol, a0);
        tmem_ld32(scol + 32, a1);
        tmem_ld32(scol + 64, a2);
        tmem_ld32(scol + 96, a3);
        tmem_ld_wait();
        reg_fence(a0);
        reg_fence(a1);
        reg_fence(a2);
        reg_fence(a3);
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          s[c] = __uint_as_float(a0[c]);
          s[32 + c] = __uint_as_float(a1[c]);
          s[64 + c] = __uint_as_float(a2[c]);
          s[96 + c] = __uint_as_float(a3[c]);
        }
      }
      if (j >= full || !ok) {
        const int lim = ok ? min(limit, it.kv_len - 1) - key0 : -1;
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c > lim) s[c] = -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int i8 = 0; i8 < 8; ++i8) mx8[i8] = s[i8];
#pragma unroll
      for (int c = 8; c < 120; c += 16) {
#pragma unroll
        for (int i8 = 0; i8 < 8; ++i8) mx8[i8] = max3(mx8[i8], s[c + i8], s[c + 8 + i8]);
      }
#pragma unroll
      for (int i8 = 0; i8 < 8; ++i8) mx8[i8] = fmaxf(mx8[i8], s[120 + i8]);
      const float m_tile =
          max3(max3(mx8[0], mx8[1], mx8[2]), max3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])) * sl2;
      // Rescale only when the row max grew by more than 2^8 (or on the first
      // finite max); otherwise keep scaling by the stale max.
      float alpha = 1.0f;
      if (m_tile > m_used + kRescaleLog2) {
        alpha = fast_exp2(m_used - m_tile);  // 0 when m_used = -inf
        m_used = m_tile;
      }
      if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        // PV_x of the previous tile completed before S_x of this one was
        // issued; the wait (already satisfied) orders its O writes here.
        if (!warp_wait(&bars[kPVDone + x], (t - 1) & 1)) {
          alive = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int h = 0; h < 4; ++h) {
          uint32_t o[32];
          tmem_ld32(ocol + h * 32, o);
          tmem_ld_wait();
          reg_fence(o);
#pragma unroll
          for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
          tmem_st32(ocol + h * 32, o);
        }
      }
      const float nm = m_used == -INFINITY ? 0.0f : -m_used;
      float sum[8];
#pragma unroll
      for (int i8 = 0; i8 < 8; ++i8) sum[i8] = 0.0f;
      {
        // keys [32 g, +32) -> packed columns [16 g, +16) of S_x
        uint32_t pk[16];
        exp32<0>(s, sl2, nm, pk, sum);
        tmem_st16(scol, pk);
        exp32<32>(s, sl2, nm, pk, sum);
        tmem_st16(scol + 16, pk);
        exp32<64>(s, sl2, nm, pk, sum);
        tmem_st16(scol + 32, pk);
        exp32<96>(s, sl2, nm, pk, sum);
        tmem_st16(scol + 48, pk);
      }
      l = l * alpha + (((sum[0] + sum[1]) + (sum[2] + sum[3])) + ((sum[4] + sum[5]) + (sum[6] + sum[7])));
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kPFull + x]);
    }
    if (!alive) break;
    // (max used, row sum) to the epilogue through a one-item slot per tile
    if (ix > 0 && !warp_wait(&bars[kStatsFree + x], (ix - 1) & 1)) break;
    // no finite score seen: the sum holds only clamped-exponent residue
    stats[x * kRows + r] = make_float2(m_used, m_used == -INFINITY ? 0.0f : l);
    mbar_arrive(&bars[kStatsFull + x]);
    ++ix;
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap qmap,
                   const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  // tiles start at the first 1024-byte boundary; the head block follows
  const uint32_t sbase = (raw_addr + 1023u) & ~1023u;
  unsigned char* tiles = smem_raw + (sbase - raw_addr);
  unsigned char* head = tiles + kTileBytes;
  const int n_items = p.n_pairs * p.batch * p.kvh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The next launch on this stream may start its set-up on SMs this grid leaves.
  asm volatile("griddepcontrol.launch_dependents;");

  uint64_t* bars = reinterpret_cast<uint64_t*>(head);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(head + kTmemSlotOff);
  Item* ring = reinterpret_cast<Item*>(head + kItemOff);
  float2* stats = reinterpret_cast<float2*>(head + kStatsOff);
  volatile int* v_real = reinterpret_cast<volatile int*>(head + kVRealOff);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kQFull + s], 1);
      mbar_init(&bars[kQFree + s], 1);
      mbar_init(&bars[kKFull + s], 1);
      mbar_init(&bars[kKEmpty + s], 1);
      mbar_init(&bars[kVFull + s], 1);
      mbar_init(&bars[kVEmpty + s], 1);
      mbar_init(&bars[kSFull + s], 1);
      mbar_init(&bars[kPFull + s], 4);
      mbar_init(&bars[kPVDone + s], 1);
      mbar_init(&bars[kODone + s], 1);
      mbar_init(&bars[kOFree + s], 4);
      mbar_init(&bars[kStatsFull + s], kRows);
      mbar_init(&bars[kStatsFree + s], kRows);
      mbar_init(&bars[kItemFull + s], 1);
      mbar_init(&bars[kItemEmpty + s], kItemReaders);
    }
    mbar_init(&bars[kDrain], 1);
    mbar_init(&bars[kPVDrain], 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp >= 12 && p.rows_used < kRows) {
    // Rows past the packed (query, head) rows are never loaded: zero them once.
    const int t = threadIdx.x - 384;
    const int per = (kRows - p.rows_used) * 16;  // 16-byte chunks per Q buffer
    for (int e = t; e < kQStages * per; e += 128) {
      const int s = e / per, rem = e - s * per;
      const int r = p.rows_used + (rem >> 4), c = rem & 15;
      st_shared_zero16(sbase + kQOff + s * kQBytes + (c >> 3) * kHalf + r * 128 + (c & 7) * 16);
    }
    fence_proxy_async_smem();
  }
  // Launched as a programmatic dependent of the previous kernel on the
  // stream: the set-up above touches only this CTA's shared memory and TMEM.
  // Wait for that kernel to complete, its writes (this stream's claim-counter
  // reset among them) visible, before any global access.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // Sequences ranked by their work (about q tiles x keys seen), heaviest
  // first, so that dynamic claiming ends with small items (the rank of each
  // sequence is the count of heavier ones; ties by index).
  int* order = nullptr;
  if (p.batch <= kMaxSorted) {
    order = reinterpret_cast<int*>(head + kOrderOff);
    float* work = reinterpret_cast<float*>(head + kWorkOff);
    for (int b = threadIdx.x; b < p.batch; b += kThreads) {
      const int q_len = p.cu_q[b + 1] - p.cu_q[b];
      const int prefix = p.kv_lens[b] - q_len;
      work[b] = (q_len > 0 && prefix >= 0)
                    ? float(p.fd_qt.div(q_len + p.qt - 1)) * (float(prefix) + 0.5f * float(q_len) + float(p.qt))
                    : 0.0f;
    }
    __syncthreads();
    for (int b = threadIdx.x; b < p.batch; b += kThreads) {
      const float wb = work[b];
      int rank = 0;
      for (int j = 0; j < p.batch; ++j) rank += (work[j] > wb) || (work[j] == wb && j < b);
      order[rank] = b;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Register split: 2 x 128 x kSoftmaxRegs + 2 x 128 x kOtherRegs = 512 x
  // 128, so every increase is met (the launcher refuses a build whose kernel
  // does not launch with kLaunchRegs). Each warpgroup executes one setmaxnreg.
  if (warp >= 4 && warp < 12) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kSoftmaxRegs));
    softmax_role(p, bars, ring, stats, tmem, warp, lane);
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kOtherRegs));
    if (warp == 0) {
      // ----------------------------------- scheduler, Q and K producer
      if (lane == 0) {
        tma_prefetch_desc(&qmap);
        tma_prefetch_desc(&kmap);
        tma_prefetch_desc(&vmap);
        int gt = 0, k_issued = 0, ixq[2] = {0, 0};
        bool alive = true;
        for (int i = 0; alive; ++i) {
          // claim the next item with queries
          int v;
          Item it;
          do {
            v = atomicAdd(p.sched, 1);
            if (v >= n_items) break;
            it = make_item(p, order, v);
            if (it.qx[0] == 0) {
              // Pairs past the sequence's queries come first in their group:
              // move the counter to the group's last (non-empty) pair if
              // nobody has claimed past this one yet.
              const int q_len = p.cu_q[it.b + 1] - it.q_begin;
              const int tiles = q_len > 0 ? p.fd_qt.div(q_len + p.qt - 1) : 0;
              const int group_end = (p.fd_npair.div(v) + 1) * p.n_pairs;
              atomicCAS(p.sched, v + 1, group_end - (tiles + 1) / 2);
            }
          } while (it.qx[0] == 0);
          const bool end = v >= n_items;
          if (end) it.b = -1;
          if (i >= 2 && !mbar_wait(&bars[kItemEmpty + (i & 1)], ((i >> 1) + 1) & 1, kErrPrefillWait)) break;
          ring[i & 1] = it;
          mbar_arrive(&bars[kItemFull + (i & 1)]);
          if (end) break;
          const int nt = item_tiles(it);
          if (nt == 0) continue;  // rows without keys: only the epilogue acts
          const int* table = p.block_table + (long long)it.b * p.table_stride;
          // K tile j of this item into the ring once both S MMAs of tile j-2 read its stage.
          auto load_k = [&](int j) -> bool {
            const int g = gt + j, st = g & 1;
            const int key0 = j * kKeys;
            const int logical = p.fd_bs.div(key0);
            const int page = table[logical];
            const bool ok = page_ok(page, p.num_blocks);
            const int trow = ok ? page * p.block_size + (key0 - logical * p.block_size) : 0;
            if (g >= kKStages && !mbar_wait(&bars[kKEmpty + st], ((g >> 1) + 1) & 1, kErrPrefillWait)) return false;
            unsigned char* kdst = tiles + kKOff + st * kKVBytes;
            if (ok) {
              mbar_arrive_expect_tx(&bars[kKFull + st], kKVBytes);
              tma_load_3d(kdst, &kmap, &bars[kKFull + st], 0, it.h, trow);
              tma_load_3d(kdst + kHalf, &kmap, &bars[kKFull + st], 64, it.h, trow);
            } else {
              mbar_arrive(&bars[kKFull + st]);
            }
            k_issued = g + 1;
            return true;
          };
          // The item's first K tile goes out before its Q tiles: its stage is
          // free two tiles before the previous item ends, the Q buffers only
          // once that item's last S MMAs have read them.
          alive = load_k(0);
#pragma unroll
          for (int x = 0; x < 2 && alive; ++x) {
            if (it.n[x] == 0) continue;
            // Q buffer x is free once the last S MMA of its previous tile completed.
            if (ixq[x] >= 1 && !mbar_wait(&bars[kQFree + x], (ixq[x] - 1) & 1, kErrPrefillWait)) {
              alive = false;
              break;
            }
            mbar_arrive_expect_tx(&bars[kQFull + x], 2u * 128u * uint32_t(p.rows_used));
            const int qy = it.h * p.group, qz = it.q_begin + it.q0[x];
            unsigned char* qdst = tiles + kQOff + x * kQBytes;
            tma_load_3d(qdst, &qmap, &bars[kQFull + x], 0, qy, qz);
            tma_load_3d(qdst + kHalf, &qmap, &bars[kQFull + x], 64, qy, qz);
            ++ixq[x];
          }
          for (int j = 1; j < nt && alive; ++j) alive = load_k(j);
          gt += nt;
        }
        // Drain: every copy this thread issued has landed before the CTA
        // exits (already true on the normal path; bounded on an error path).
#pragma unroll
        for (int s = 0; s < 2; ++s) {
          if (k_issued > s) mbar_wait(&bars[kKFull + s], ((k_issued - 1 - s) >> 1) & 1, kErrPrefillWait);
          if (ixq[s] > 0) mbar_wait(&bars[kQFull + s], (ixq[s] - 1) & 1, kErrPrefillWait);
        }
      }
    } else if (warp == 3) {
      // --------------------------------------------------- V producer
      if (lane == 0) {
        tma_prefetch_desc(&vmap);
        int gt = 0, v_issued = 0;
        bool alive = true;
        Item it;
        for (int i = 0; alive && take_item(bars, ring, i, false, it); ++i) {
          const int nt = item_tiles(it);
          const int* table = p.block_table + (long long)it.b * p.table_stride;
          for (int j = 0; j < nt; ++j) {
            const int g = gt + j, st = g & 1;
            const int key0 = j * kKeys;
            const int logical = p.fd_bs.div(key0);
            const int page = table[logical];
            const bool ok = page_ok(page, p.num_blocks);
            const int trow = ok ? page * p.block_size + (key0 - logical * p.block_size) : 0;
            if (g >= kVStages && !mbar_wait(&bars[kVEmpty + st], ((g >> 1) + 1) & 1, kErrPrefillWait)) {
              alive = false;
              break;
            }
            unsigned char* vdst = tiles + kVOff + st * kKVBytes;
            // keys of the tile that are real (the fixer zeroes the rest); the
            // arrival below releases the store to the fixer's wait
            v_real[st] = ok ? min(kKeys, it.kv_len - key0) : 0;
            if (ok) {
              mbar_arrive_expect_tx(&bars[kVFull + st], kKVBytes);
              tma_load_3d(vdst, &vmap, &bars[kVFull + st], 0, it.h, trow);
              tma_load_3d(vdst + kHalf, &vmap, &bars[kVFull + st], 64, it.h, trow);
            } else {
              mbar_arrive(&bars[kVFull + st]);
            }
            v_issued = g + 1;
          }
          gt += nt;
        }
#pragma unroll
        for (int s = 0; s < 2; ++s)
          if (v_issued > s) mbar_wait(&bars[kVFull + s], ((v_issued - 1 - s) >> 1) & 1, kErrPrefillWait);
      }
    } else if (warp == 1) {
      // --------------------------------------------------- S MMA issuer
      // Per KV tile j: S_A = Q_A K_j^T, then S_B = Q_B K_j^T. S_x is single-
      // buffered, so S_x for tile j waits for PV_x of its previous tile (the
      // P that PV read sits in the same TMEM columns).
      if (lane == 0) {
        int gt = 0, tx[2] = {0, 0}, ixq[2] = {0, 0};
        bool alive = true;
        // Descriptors of Q buffer 0 and K stage 0; buffers/stages are 2048 16-byte units apart.
        const uint64_t qd = sw128_desc(sbase + kQOff, 16, 1024), kd = sw128_desc(sbase + kKOff, 16, 1024);
        const uint32_t q_lo = uint32_t(qd), q_hi = uint32_t(qd >> 32), k_lo = uint32_t(kd), k_hi = uint32_t(kd >> 32);
        static_assert(kQBytes == kKVBytes && kKVBytes >> 4 == 2048, "stage stride in descriptor units");
        Item it;
        for (int i = 0; alive && take_item(bars, ring, i, false, it); ++i) {
          const int nt = item_tiles(it);
          for (int j = 0; j < nt && alive; ++j) {
            const int g = gt + j, ks = g & 1;
            alive = mbar_wait(&bars[kKFull + ks], (g >> 1) & 1, kErrPrefillWait);
            const uint32_t kb = k_lo + uint32_t(ks) * 2048u;
#pragma unroll
            for (int x = 0; x < 2 && alive; ++x) {
              if (j >= it.n[x]) continue;
              if (j == 0) alive = mbar_wait(&bars[kQFull + x], ixq[x] & 1, kErrPrefillWait);
              if (alive && tx[x] >= 1) alive = mbar_wait(&bars[kPVDone + x], (tx[x] - 1) & 1, kErrPrefillWait);
              if (!alive) break;
              tc_fence_after();
              const uint32_t qa = q_lo + uint32_t(x) * 2048u, sd = tmem + kSCol + x * kKeys;
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                const uint32_t off = uint32_t((kk >> 2) * kHalf + (kk & 3) * 32) >> 4;
                umma_ss(sd, qa + off, q_hi, kb + off, k_hi, kIdescS, kk > 0 ? 1u : 0u);
              }
              umma_commit(&bars[kSFull + x]);
              if (j == it.n[x] - 1) {
                umma_commit(&bars[kQFree + x]);
                ++ixq[x];
              }
              ++tx[x];
            }
            if (alive) umma_commit(&bars[kKEmpty + ks]);
          }
          gt += nt;
        }
        // every MMA issued by this thread completes before TMEM is freed
        umma_commit(&bars[kDrain]);
        mbar_wait(&bars[kDrain], 0, kErrPrefillWait);
      }
    } else if (warp == 2) {
      // ---------------------------------------- V fixer and PV issuer
      // Fixes V_j (zeroes rows that are not real keys: past kv_len or an
      // invalid page, so P ~ 0 never meets a non-finite cache value), then
      // lane 0 issues O_A += P_A V_j and O_B += P_B V_j (the S MMAs come from
      // warp 1: two issuing threads). A tile's first PV also waits for the
      // epilogue's read of that tile's previous O.
      int gt = 0, tx[2] = {0, 0}, ixo[2] = {0, 0};
      bool alive = true;
      const uint64_t vd = sw128_desc(sbase + kVOff, kHalf, 1024);
      const uint32_t v_lo = uint32_t(vd), v_hi = uint32_t(vd >> 32);
      Item it;
      for (int i = 0; alive && take_item(bars, ring, i, true, it); ++i) {
        const int nt = item_tiles(it);
        for (int j = 0; j < nt; ++j) {
          const int g = gt + j, st = g & 1;
          if (!warp_wait(&bars[kVFull + st], (g >> 1) & 1)) {
            alive = false;
            break;
          }
          const int real = v_real[st];  // written by the V producer before its arrival
          if (real < kKeys) {
            const uint32_t vbase = sbase + kVOff + st * kKVBytes;
            for (int e = lane; e < (kKeys - real) * 16; e += 32) {
              const int row = real + (e >> 4), c = e & 15;
              st_shared_zero16(vbase + (c >> 3) * kHalf + row * 128 + (c & 7) * 16);
            }
            fence_proxy_async_smem();
          }
          __syncwarp();
          bool ok_pv = true;
          if (lane == 0) {
            const uint32_t vb = v_lo + uint32_t(st) * 2048u;
#pragma unroll
            for (int x = 0; x < 2 && ok_pv; ++x) {
              if (j >= it.n[x]) continue;
              if (j == 0 && ixo[x] > 0) ok_pv = mbar_wait(&bars[kOFree + x], (ixo[x] - 1) & 1, kErrPrefillWait);
              if (ok_pv) ok_pv = mbar_wait(&bars[kPFull + x], tx[x] & 1, kErrPrefillWait);
              if (!ok_pv) break;
              tc_fence_after();
              const uint32_t pa = tmem + kSCol + x * kKeys, od = tmem + kOCol + x * kKeys;
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                // P: 16 keys = 8 packed columns; V: 16 keys = 2048 bytes of rows
                umma_ts(od, pa + kk * 8, vb + kk * 128, v_hi, kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
              }
              umma_commit(&bars[kPVDone + x]);
              if (j == it.n[x] - 1) {
                umma_commit(&bars[kODone + x]);
                ++ixo[x];
              }
              ++tx[x];
            }
            if (ok_pv) umma_commit(&bars[kVEmpty + st]);
          }
          if (!__shfl_sync(0xffffffffu, ok_pv, 0)) {
            alive = false;
            break;
          }
        }
        gt += nt;
      }
      if (lane == 0) {
        // every PV MMA completes before TMEM is freed
        umma_commit(&bars[kPVDrain]);
        mbar_wait(&bars[kPVDrain], 0, kErrPrefillWait);
      }
    } else if (warp >= 12) {
      // ------------------------------------------------------- epilogue
      // O_x / l -> BF16 rows and the LSE for tile A, then tile B; frees O_x
      // for its next tile as soon as it is read.
      const int quad = warp & 3;
      const int r = quad * 32 + lane;
      const uint32_t lane_base = tmem + (uint32_t(quad * 32) << 16);
      const int rq = r / p.group;
      const int rh = r - rq * p.group;
      int ixo[2] = {0, 0};
      bool alive = true;
      Item it;
      for (int i = 0; alive && take_item(bars, ring, i, true, it); ++i) {
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (it.qx[x] == 0) continue;
          const int qpos = it.q0[x] + rq;
          const bool valid_row = r < p.rows_used && rq < it.qx[x] && qpos < p.max_q;
          const int head = it.h * p.group + rh;
          __nv_bfloat16* dst = p.out + (((long long)it.q_begin + qpos) * p.qh + head) * 128;
          float* lse_dst = p.lse ? p.lse + ((long long)it.b * p.qh + head) * p.max_q + qpos : nullptr;
          if (it.n[x] == 0) {
            // No visible keys (invalid context): zero rows, -inf LSE.
            if (valid_row) {
              for (int d = 0; d < 128; d += 8) *reinterpret_cast<uint4*>(dst + d) = make_uint4(0, 0, 0, 0);
              if (lse_dst) *lse_dst = -INFINITY;
            }
            continue;
          }
          if (!warp_wait(&bars[kStatsFull + x], ixo[x] & 1)) {
            alive = false;
            break;
          }
          const float2 ml = stats[x * kRows + r];
          mbar_arrive(&bars[kStatsFree + x]);
          if (!warp_wait(&bars[kODone + x], ixo[x] & 1)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const float l = ml.y;
          const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll 1
          for (int h = 0; h < 8; ++h) {  // 16 columns at a time (this warpgroup runs on kOtherRegs)
            uint32_t o[16];
            tmem_ld16(lane_base + kOCol + x * kKeys + h * 16, o);
            tmem_ld_wait();
            reg_fence(o);
            if (h == 7) {
              // O_x is read: free it for the next item's first PV before the last stores.
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&bars[kOFree + x]);
            }
            if (valid_row) {
#pragma unroll
              for (int vv = 0; vv < 2; ++vv) {
                const uint32_t* src = o + 8 * vv;
                uint4 w;
                w.x = pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
                w.y = pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
                w.z = pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
                w.w = pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
                *reinterpret_cast<uint4*>(dst + h * 16 + vv * 8) = w;
              }
            }
          }
          if (valid_row && lse_dst) {
            const float m_out = ml.x == -INFINITY ? 0.0f : ml.x;
            *lse_dst = l > 0.0f ? (m_out + fast_log2(l)) * kLn2 : -INFINITY;
          }
          ++ixo[x];
        }
      }
    }
  }  // register split

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
    if (atomicAdd(p.sched + 1, 1) == int(gridDim.x) - 1) {
      atomicExch(p.sched, 0);
      atomicExch(p.sched + 1, 0);
    }
  }
}

// Claim counters {next item, CTAs finished}, one pair per stream that
// launches the prefill (a launch leaves its pair at zero when it ends).
__device__ int g_prefill_sched[64][2];

// Pair for (stream, context): streams get their own pair in order of first
// use; past 64 streams pairs are shared by hash, and launches sharing a pair
// must not overlap in time.
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
    *err = cudaGetSymbolAddress(&ptr, g_prefill_sched);
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

}  // namespace prefill_detail

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream) {
  using namespace prefill_detail;
  const int group = a.qh / a.kvh;
  // Up to 128 query heads per kv head: a 128-row query tile holds 128 / group
  // queries of the group (at least one).
  if (group < 1 || group > kRows || a.batch > 65535 || a.kvh > 65535) return cudaErrorNotSupported;
  const int qt = kRows / group;
  // Every sequence within one query tile (chunked prefill of short chunks):
  // tile B of every pair would be empty, so one tile per item runs faster.
  if (a.max_q <= qt) return launch_prefill_tile(a, stream);
  PrefillParams p{};
  p.cu_q = a.cu_q;
  p.kv_lens = a.kv_lens;
  p.block_table = a.block_table;
  p.out = static_cast<__nv_bfloat16*>(const_cast<void*>(a.out));
  p.lse = a.lse;
  p.batch = a.batch;
  p.max_q = a.max_q;
  p.qh = a.qh;
  p.kvh = a.kvh;
  p.group = group;
  p.qt = qt;
  p.rows_used = qt * group;
  p.block_size = a.block_size;
  p.table_stride = a.table_stride;
  p.num_blocks = a.num_blocks;
  p.scale_log2 = 1.4426950408889634f / 11.313708498984761f;

  CUtensorMap qmap, kmap, vmap;
  {
    const uint64_t dims[3] = {128, uint64_t(a.qh), uint64_t(a.total_q)};
    const uint64_t strides[2] = {256, uint64_t(a.qh) * 256};
    const uint32_t box[3] = {64, uint32_t(group), uint32_t(qt)};
    if (make_map_3d(a.q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, &qmap)) return cudaErrorInvalidValue;
  }
  {
    const uint64_t dims[3] = {128, uint64_t(a.kvh), uint64_t(a.num_blocks) * uint64_t(a.block_size)};
    const uint64_t strides[2] = {256, uint64_t(a.kvh) * 256};
    const uint32_t box[3] = {64, 1, uint32_t(kKeys)};
    if (make_map_3d(a.k, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, &kmap)) return cudaErrorInvalidValue;
    if (make_map_3d(a.v, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, &vmap)) return cudaErrorInvalidValue;
  }
  static unsigned configured[kContextSlots] = {};
  cudaError_t e = once_per_context(configured, [] {
    cudaError_t r = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (r != cudaSuccess) return r;
    // The in-kernel register split assumes exactly kLaunchRegs a thread at
    // launch; with fewer, a setmaxnreg.inc would wait for registers forever.
    cudaFuncAttributes fa{};
    r = cudaFuncGetAttributes(&fa, prefill_kernel);
    if (r != cudaSuccess) return r;
    return fa.numRegs == kLaunchRegs ? cudaSuccess : cudaErrorInvalidKernelImage;
  });
  if (e != cudaSuccess) return e;
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static int sm_count[64] = {};
  if (!sm_count[dev & 63]) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sm_count[dev & 63] = n;
  }
  p.sched = sched_pair(stream, &e);
  if (!p.sched) return e;
  p.n_qtiles = (a.max_q + qt - 1) / qt;
  p.n_pairs = (p.n_qtiles + 1) / 2;
  p.fd_npair = FastDiv::make(p.n_pairs > 0 ? p.n_pairs : 1);
  p.fd_kvh = FastDiv::make(a.kvh);
  p.fd_qt = FastDiv::make(qt);
  p.fd_bs = FastDiv::make(a.block_size);
  const long long items = (long long)p.n_pairs * a.batch * a.kvh;
  if (items > 0x7fffffffLL) return cudaErrorNotSupported;
  const int grid = int(items < sm_count[dev & 63] ? items : sm_count[dev & 63]);
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
  return cudaLaunchKernelEx(&cfg, prefill_kernel, p, qmap, kmap, vmap);
}

}  // namespace nvb
