// Varlen / chunked causal prefill over the paged KV cache on tcgen05 tensor
// cores (sm_100a): the one-query-tile-per-item kernel. launch_prefill
// (prefill.cu) sends it launches whose sequences all fit one 128-row query
// tile (chunked prefill of short chunks), where prefill.cu's pairs of query
// tiles would leave one tile of every pair empty.
//
// Replaces the reference's prefill paths: FA2's paged split-KV kernel with
// num_splits = 1 and a bottom-right causal mask (SM80 mma.sync, launched from
// kernels/flash_native/flash_native.cu:102-112) and the native ordered kernel
// (kernels/kernels.cu:288-354, one CTA per query row). The causal rule is the
// reference's: query i of a q_len-query group sees keys
// [0, kv_len - q_len + i] (src/model.rs:1170-1188, smoke.cu:58).
//
// Work item: one 128-row query tile of one (sequence, kv head). Rows pack the
// GQA group: row r is (query q0 + r / G, head h*G + r % G), so each K/V tile
// serves every query head of the group. Per 128-key KV tile t:
//
//   S_t = Q K_t^T   tcgen05.mma kind::f16, M=128 N=128 K=128 (8 x K16), A and B
//                   from 128B-swizzled shared memory, D in TMEM (FP32)
//   P_t = exp2(S_t * scale*log2e - m)   two softmax warpgroups, each thread
//                   one row and one half (64 keys) of the tile; P written back
//                   over S_t in TMEM as packed BF16
//   O  += P_t V_t   tcgen05.mma M=128 N=128 K=128, A (P) read from TMEM, V an
//                   MN-major B operand in shared memory, O in TMEM
//
// S/P is triple-buffered in TMEM (columns 0, 128, 256; O at 384): S_{t+1} is
// issued as soon as PV_{t-2} has released its buffer, so the tensor core
// computes the next scores while the softmax works on the current ones and
// the per-tile work of the tensor core (1024 cycles at M=N=K=128) overlaps the
// softmax (~2,000 cycles a tile for the two warps of an SMSP, of which the
// exponentials take ~1,100 on the 16-per-clock MUFU unit).
//
// Roles (16 warps, one CTA per SM):
//   warp 0      claims items (global counter, heaviest first), publishes each
//               to the CTA through a two-slot ring, loads Q (two buffers) and
//               the K tiles (two-stage ring) with TMA: 3-D maps over [tokens,
//               kv_heads, 128], 64-element 128-byte-swizzled boxes; a 128-key
//               tile never crosses a page since block_size is a multiple of 256
//   warp 1      TMEM owner; one thread issues the S MMAs and their commits
//   warp 2      V fixer and PV issuer: zeroes V rows that are not real keys
//               (past kv_len or an invalid page) so P ~ 0 never meets a
//               non-finite cache value, then one thread issues that tile's
//               PV MMAs once P is in TMEM (two issuing threads: neither the
//               S nor the PV stream waits behind the other's barriers)
//   warp 3      loads the V tiles (two-stage ring)
//   warps 4-7   softmax of keys 0-63 of each tile; warps 8-11 keys 64-127. The
//               two halves of a row agree on its max through shared memory and
//               a per-quadrant mbarrier (no bar.sync: every wait is bounded)
//   warps 12-15 epilogue: O / l -> BF16 rows and the LSE, from row statistics
//               handed over in shared memory; frees O for the next item
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

namespace prefill_tile_detail {

using namespace prefill_common;

constexpr int kRows = 128;                   // query rows per item (TMEM lanes)
constexpr int kKeys = 128;                   // keys per KV tile
constexpr int kHalf = 128 * 128;             // 128 rows x 64 BF16 (one 128-byte swizzle column)
constexpr int kQBytes = 2 * kHalf;           // Q tile 128 x 128 BF16
constexpr int kKVBytes = 2 * kHalf;          // K or V tile 128 x 128 BF16
constexpr int kQStages = 2, kKStages = 2, kVStages = 2;
constexpr int kSBufs = 3;                    // S/P buffers in TMEM
constexpr int kThreads = 512;
constexpr int kTmemCols = 512;
constexpr int kOCol = 384;
constexpr float kLn2 = 0.693147180559945309f;
constexpr float kRescaleLog2 = 8.0f;         // lazy rescale threshold (P <= 2^8)

enum Bar {
  kQFull = 0, kQFree = 2, kKFull = 4, kKEmpty = 6, kVFull = 8, kPVDrain = 10, kVEmpty = 12,  // [2]
  kSFull = 14, kPVDone = 17, kPFull = 20,                                                  // [3]: per S buffer
  kODone = 23, kOFree = 24, kStatsFull = 25, kStatsFree = 26,
  kXchg = 27,                                                                              // [4]: per TMEM quadrant
  kItemFull = 31, kItemEmpty = 33,                                                         // [2]
  kDrain = 35, kNumBars = 36
};
// Readers of each published item: V producer, MMA issuer, V fixer (one
// arrival each) and the 8 softmax + 4 epilogue warps (one per warp).
constexpr int kItemReaders = 15;
constexpr int kTmemSlotOff = kNumBars * 8;
constexpr int kItemOff = 320;                               // Item [2] (the published-item ring)
constexpr int kItemBytes = 64;
constexpr int kStatsOff = 512;                              // float2 [128]: row max used, row sum
constexpr int kXOff = kStatsOff + kRows * 8;                // float [2 slots][2 halves][128]
constexpr int kMaxSorted = 1024;                            // batches up to this size are claimed by work
constexpr int kOrderOff = kXOff + 2 * 2 * kRows * 4;        // int [kMaxSorted]: sequences, heaviest first
constexpr int kWorkOff = kOrderOff + kMaxSorted * 4;        // float [kMaxSorted]: each sequence's work
constexpr int kHeadBytes = kWorkOff + kMaxSorted * 4;
constexpr int kQOff = 0;                                    // offsets from the 1 KB aligned tile base
constexpr int kKOff = kQOff + kQStages * kQBytes;
constexpr int kVOff = kKOff + kKStages * kKVBytes;
constexpr int kTileBytes = kVOff + kVStages * kKVBytes;     // 192 KB
constexpr int kSmemBytes = kTileBytes + kHeadBytes + 1024;  // + worst-case alignment pad
static_assert(kTmemSlotOff + 4 <= kItemOff && kItemOff + 2 * kItemBytes <= kStatsOff, "head layout overlaps");
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
  FastDiv fd_nqt, fd_kvh, fd_qt, fd_bs;  // by n_qtiles, kvh, qt, block_size
};

// One 128-row query tile of one (sequence, kv head): the work item of the
// persistent loop. Virtual items are grouped by (sequence, kv head), longest
// causal tile first within a group, so the CTAs running at one time share a
// few groups' K/V in L2; the sequences come heaviest first (ranked at kernel
// start for batches up to kMaxSorted) and CTAs claim items from a global
// counter (dynamic load balancing), so the last claims are small ones.
struct Item {
  int b, h, q_begin, q0, kv_len, prefix;
  int qx;       // queries in the tile
  int key_end;  // keys its last query sees
  int n;        // KV tiles it visits
  int full;     // leading KV tiles that every row sees whole
};
static_assert(sizeof(Item) <= kItemBytes, "item ring slot too small");

// `order` (or null): sequence of each rank, heaviest first.
__device__ __forceinline__ Item make_item(const PrefillParams& p, const int* order, int v) {
  Item it;
  const int group = p.fd_nqt.div(v);
  const int tile = p.n_qtiles - 1 - (v - group * p.n_qtiles);
  const int rank = p.fd_kvh.div(group);
  it.b = order ? order[rank] : rank;
  it.h = group - rank * p.kvh;
  it.q_begin = p.cu_q[it.b];
  const int q_len = p.cu_q[it.b + 1] - it.q_begin;
  it.q0 = tile * p.qt;
  it.qx = max(0, min(p.qt, q_len - it.q0));
  it.kv_len = it.qx > 0 ? p.kv_lens[it.b] : 0;
  it.prefix = it.kv_len - q_len;
  // A context longer than the page table, or shorter than its query group,
  // is invalid input: such rows get zero output (as decode does).
  const bool seq_ok = it.qx > 0 && it.prefix >= 0 && (long long)it.kv_len <= (long long)p.table_stride * p.block_size;
  it.key_end = seq_ok ? min(it.kv_len, it.prefix + it.q0 + it.qx) : 0;
  it.n = (it.key_end + kKeys - 1) / kKeys;
  it.full = seq_ok ? min(it.kv_len, it.prefix + it.q0 + 1) / kKeys : 0;
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

__global__ void __launch_bounds__(kThreads, 1)
    prefill_tile_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap qmap,
                   const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  // tiles start at the first 1024-byte boundary; the head block follows
  const uint32_t sbase = (raw_addr + 1023u) & ~1023u;
  unsigned char* tiles = smem_raw + (sbase - raw_addr);
  unsigned char* head = tiles + kTileBytes;
  const int n_items = p.n_qtiles * p.batch * p.kvh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The next launch on this stream may start its set-up on SMs this grid leaves.
  asm volatile("griddepcontrol.launch_dependents;");

  uint64_t* bars = reinterpret_cast<uint64_t*>(head);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(head + kTmemSlotOff);
  Item* ring = reinterpret_cast<Item*>(head + kItemOff);
  float2* stats = reinterpret_cast<float2*>(head + kStatsOff);
  float* xch = reinterpret_cast<float*>(head + kXOff);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kQFull + s], 1);
      mbar_init(&bars[kQFree + s], 1);
      mbar_init(&bars[kKFull + s], 1);
      mbar_init(&bars[kKEmpty + s], 1);
      mbar_init(&bars[kVFull + s], 1);
      mbar_init(&bars[kPVDrain + s], 1);
      mbar_init(&bars[kVEmpty + s], 1);
      mbar_init(&bars[kItemFull + s], 1);
      mbar_init(&bars[kItemEmpty + s], kItemReaders);
    }
#pragma unroll
    for (int b = 0; b < kSBufs; ++b) {
      mbar_init(&bars[kSFull + b], 1);
      mbar_init(&bars[kPVDone + b], 1);
      mbar_init(&bars[kPFull + b], 8);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) mbar_init(&bars[kXchg + q], 64);
    mbar_init(&bars[kODone], 1);
    mbar_init(&bars[kOFree], 4);
    mbar_init(&bars[kStatsFull], kRows);
    mbar_init(&bars[kStatsFree], kRows);
    mbar_init(&bars[kDrain], 1);
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

  if (warp == 0) {
    // ------------------------------------- scheduler, Q and K producer
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      int gt = 0, ix = 0, k_issued = 0;
      bool alive = true;
      for (int i = 0; alive; ++i) {
        // claim the next item that has queries
        int v;
        Item it;
        do {
          v = atomicAdd(p.sched, 1);
          if (v >= n_items) break;
          it = make_item(p, order, v);
          if (it.qx == 0) {
            // Tiles past the sequence's queries come first in their group:
            // move the counter to the group's last (non-empty) tile if nobody
            // has claimed past this one yet.
            const int q_len = p.cu_q[it.b + 1] - it.q_begin;
            const int tiles = q_len > 0 ? p.fd_qt.div(q_len + p.qt - 1) : 0;
            const int group_end = (p.fd_nqt.div(v) + 1) * p.n_qtiles;
            atomicCAS(p.sched, v + 1, group_end - tiles);
          }
        } while (it.qx == 0);
        const bool end = v >= n_items;
        if (end) it.b = -1;
        if (i >= 2 && !mbar_wait(&bars[kItemEmpty + (i & 1)], ((i >> 1) + 1) & 1, kErrPrefillWait)) break;
        ring[i & 1] = it;
        mbar_arrive(&bars[kItemFull + (i & 1)]);
        if (end) break;
        if (it.n == 0) continue;  // rows without keys: only the epilogue acts
        const int qs = ix & 1;
        // Q buffer qs is free once the last S MMA of item ix-2 completed.
        if (ix >= 2 && !mbar_wait(&bars[kQFree + qs], ((ix >> 1) + 1) & 1, kErrPrefillWait)) break;
        mbar_arrive_expect_tx(&bars[kQFull + qs], 2u * 128u * uint32_t(p.rows_used));
        {
          const int qy = it.h * p.group, qz = it.q_begin + it.q0;
          unsigned char* qdst = tiles + kQOff + qs * kQBytes;
          tma_load_3d(qdst, &qmap, &bars[kQFull + qs], 0, qy, qz);
          tma_load_3d(qdst + kHalf, &qmap, &bars[kQFull + qs], 64, qy, qz);
        }
        ++ix;
        const int* table = p.block_table + (long long)it.b * p.table_stride;
        for (int j = 0; j < it.n; ++j) {
          const int g = gt + j, st = g & 1;
          const int key0 = j * kKeys;
          const int logical = p.fd_bs.div(key0);
          const int page = table[logical];
          const bool ok = page_ok(page, p.num_blocks);
          const int trow = ok ? page * p.block_size + (key0 - logical * p.block_size) : 0;
          if (g >= kKStages && !mbar_wait(&bars[kKEmpty + st], ((g >> 1) + 1) & 1, kErrPrefillWait)) {
            alive = false;
            break;
          }
          unsigned char* kdst = tiles + kKOff + st * kKVBytes;
          if (ok) {
            mbar_arrive_expect_tx(&bars[kKFull + st], kKVBytes);
            tma_load_3d(kdst, &kmap, &bars[kKFull + st], 0, it.h, trow);
            tma_load_3d(kdst + kHalf, &kmap, &bars[kKFull + st], 64, it.h, trow);
          } else {
            mbar_arrive(&bars[kKFull + st]);
          }
          k_issued = g + 1;
        }
        gt += it.n;
      }
      // Drain: every copy this thread issued has landed before the CTA exits
      // (already true on the normal path; bounded on an error path).
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        if (k_issued > s) mbar_wait(&bars[kKFull + s], ((k_issued - 1 - s) >> 1) & 1, kErrPrefillWait);
        if (ix > s) mbar_wait(&bars[kQFull + s], ((ix - 1 - s) >> 1) & 1, kErrPrefillWait);
      }
    }
  } else if (warp == 3) {
    // ------------------------------------------------------- V producer
    if (lane == 0) {
      tma_prefetch_desc(&vmap);
      int gt = 0, v_issued = 0;
      bool alive = true;
      Item it;
      for (int i = 0; alive && take_item(bars, ring, i, false, it); ++i) {
        if (it.n == 0) continue;
        const int* table = p.block_table + (long long)it.b * p.table_stride;
        for (int j = 0; j < it.n; ++j) {
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
          if (ok) {
            mbar_arrive_expect_tx(&bars[kVFull + st], kKVBytes);
            tma_load_3d(vdst, &vmap, &bars[kVFull + st], 0, it.h, trow);
            tma_load_3d(vdst + kHalf, &vmap, &bars[kVFull + st], 64, it.h, trow);
          } else {
            mbar_arrive(&bars[kVFull + st]);
          }
          v_issued = g + 1;
        }
        gt += it.n;
      }
#pragma unroll
      for (int s = 0; s < 2; ++s)
        if (v_issued > s) mbar_wait(&bars[kVFull + s], ((v_issued - 1 - s) >> 1) & 1, kErrPrefillWait);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int gt = 0, ix = 0;  // tiles and items (with keys) so far
      bool alive = true;
      // Descriptors of stage 0 of Q, K and V; stages are 2048 16-byte units apart.
      const uint64_t qd = sw128_desc(sbase + kQOff, 16, 1024), kd = sw128_desc(sbase + kKOff, 16, 1024);
      const uint32_t q_lo = uint32_t(qd), q_hi = uint32_t(qd >> 32), k_lo = uint32_t(kd), k_hi = uint32_t(kd >> 32);
      static_assert(kQBytes == kKVBytes && kKVBytes >> 4 == 2048, "stage stride in descriptor units");
      Item it;
      for (int i = 0; alive && take_item(bars, ring, i, false, it); ++i) {
        if (it.n == 0) continue;
        const int qs = ix & 1;
        for (int j = 0; j < it.n && alive; ++j) {
          const int t = gt + j, ks = t & 1, buf = t % kSBufs;
          alive = mbar_wait(&bars[kKFull + ks], (t >> 1) & 1, kErrPrefillWait);
          if (alive && j == 0) alive = mbar_wait(&bars[kQFull + qs], (ix >> 1) & 1, kErrPrefillWait);
          // buffer `buf` last held P_{t-3}: PV_{t-3} must have read it
          if (alive && t >= kSBufs)
            alive = mbar_wait(&bars[kPVDone + buf], ((t - kSBufs) / kSBufs) & 1, kErrPrefillWait);
          if (!alive) break;
          tc_fence_after();
          const uint32_t qa = q_lo + uint32_t(qs) * 2048u, kb = k_lo + uint32_t(ks) * 2048u, sd = tmem + buf * kKeys;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = uint32_t((kk >> 2) * kHalf + (kk & 3) * 32) >> 4;
            umma_ss(sd, qa + off, q_hi, kb + off, k_hi, kIdescS, kk > 0 ? 1u : 0u);
          }
          umma_commit(&bars[kSFull + buf]);
          umma_commit(&bars[kKEmpty + ks]);
          if (j == it.n - 1) umma_commit(&bars[kQFree + qs]);
        }
        if (!alive) break;
        ++ix;
        gt += it.n;
      }
      // every MMA issued by this thread completes before TMEM is freed
      umma_commit(&bars[kDrain]);
      mbar_wait(&bars[kDrain], 0, kErrPrefillWait);
    }
  } else if (warp == 2) {
    // ------------------------------------------- V fixer and PV issuer
    // Fixes V_t, then lane 0 issues O += P_t V_t (the S MMAs come from warp
    // 1: two issuing threads, so neither stream waits behind the other's
    // barriers). The item's first PV also waits for the epilogue's read of the
    // previous item's O.
    int gt = 0, ix = 0;
    bool alive = true;
    const uint64_t vd = sw128_desc(sbase + kVOff, kHalf, 1024);
    const uint32_t v_lo = uint32_t(vd), v_hi = uint32_t(vd >> 32);
    Item it;
    for (int i = 0; alive && take_item(bars, ring, i, true, it); ++i) {
      if (it.n == 0) continue;
      const int* table = p.block_table + (long long)it.b * p.table_stride;
      for (int j = 0; j < it.n; ++j) {
        const int g = gt + j, st = g & 1;
        const int key0 = j * kKeys;
        const bool ok = page_ok(table[p.fd_bs.div(key0)], p.num_blocks);
        const int real = ok ? min(kKeys, it.kv_len - key0) : 0;
        if (!warp_wait(&bars[kVFull + st], (g >> 1) & 1)) {
          alive = false;
          break;
        }
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
          const int buf = g % kSBufs;
          if (j == 0 && ix > 0) ok_pv = mbar_wait(&bars[kOFree], (ix - 1) & 1, kErrPrefillWait);
          if (ok_pv) ok_pv = mbar_wait(&bars[kPFull + buf], (g / kSBufs) & 1, kErrPrefillWait);
          if (ok_pv) {
            tc_fence_after();
            const uint32_t vb = v_lo + uint32_t(st) * 2048u, pa = tmem + buf * kKeys;
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              // P: 16 keys = 8 packed columns; V: 16 keys = 2048 bytes of rows
              umma_ts(tmem + kOCol, pa + kk * 8, vb + kk * 128, v_hi, kIdescPV, (j > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(&bars[kPVDone + buf]);
            umma_commit(&bars[kVEmpty + st]);
            if (j == it.n - 1) umma_commit(&bars[kODone]);
          }
        }
        if (!__shfl_sync(0xffffffffu, ok_pv, 0)) {
          alive = false;
          break;
        }
      }
      ++ix;
      gt += it.n;
    }
    if (lane == 0) {
      // every PV MMA completes before TMEM is freed
      umma_commit(&bars[kPVDrain]);
      mbar_wait(&bars[kPVDrain], 0, kErrPrefillWait);
    }
  } else if (warp < 12) {
    // ---------------------------------------------------------- softmax
    const int hf = (warp - 4) >> 2;  // which 64 keys of each tile
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // TMEM lane = packed row
    const uint32_t lane_base = tmem + (uint32_t(quad * 32) << 16);
    const int rq = r / p.group;
    const float sl2 = p.scale_log2;
    int t = 0, ix = 0, xc = 0;  // tiles, items with keys, max exchanges
    bool alive = true;
    // Exchange one value per row with the other half (same TMEM quadrant).
    auto exchange = [&](float mine, float& other) -> bool {
      float* slot = xch + (xc & 1) * 2 * kRows;
      slot[hf * kRows + r] = mine;
      mbar_arrive(&bars[kXchg + quad]);
      if (!warp_wait(&bars[kXchg + quad], xc & 1)) return false;
      other = slot[(1 - hf) * kRows + r];
      ++xc;
      return true;
    };
    Item it;
    for (int i = 0; alive && take_item(bars, ring, i, true, it); ++i) {
      if (it.n == 0) continue;
      const int* table = p.block_table + (long long)it.b * p.table_stride;
      const bool valid_row = r < p.rows_used && rq < it.qx;
      const int limit = valid_row ? it.prefix + it.q0 + rq : it.key_end - 1;  // last visible key
      float m_used = -INFINITY, l = 0.0f;  // running max the probabilities are scaled by
      for (int j = 0; j < it.n; ++j, ++t) {
        const int buf = t % kSBufs;
        const int key0 = j * kKeys;
        const bool ok = page_ok(table[p.fd_bs.div(key0)], p.num_blocks);
        if (!warp_wait(&bars[kSFull + buf], (t / kSBufs) & 1)) {
          alive = false;
          break;
        }
        tc_fence_after();
        const uint32_t scol = lane_base + buf * kKeys;
        float s[64];
        {
          uint32_t a0[32], a1[32];
          tmem_ld32(scol + hf * 64, a0);
          tmem_ld32(scol + hf * 64 + 32, a1);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            s[c] = __uint_as_float(a0[c]);
            s[32 + c] = __uint_as_float(a1[c]);
          }
        }
        if (j >= it.full || !ok) {
          const int lim = (ok ? min(limit, it.kv_len - 1) - key0 : -1) - hf * 64;
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c > lim) s[c] = -INFINITY;
        }
        float mx8[8];
#pragma unroll
        for (int i8 = 0; i8 < 8; ++i8) mx8[i8] = s[i8];
#pragma unroll
        for (int c = 8; c < 56; c += 16) {
#pragma unroll
          for (int i8 = 0; i8 < 8; ++i8) mx8[i8] = max3(mx8[i8], s[c + i8], s[c + 8 + i8]);
        }
#pragma unroll
        for (int i8 = 0; i8 < 8; ++i8) mx8[i8] = fmaxf(mx8[i8], s[56 + i8]);
        const float pm = max3(max3(mx8[0], mx8[1], mx8[2]), max3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        // The other half may overwrite S columns this half has read (its P
        // store) once both have arrived.
        tc_fence_before();
        float om;
        if (!exchange(pm, om)) {
          alive = false;
          break;
        }
        tc_fence_after();
        const float m_tile = fmaxf(pm, om) * sl2;
        // Rescale only when the row max grew by more than 2^8 (or on the
        // first finite max); otherwise keep scaling by the stale max. Both
        // halves see the same values, so they decide alike.
        float alpha = 1.0f;
        if (m_tile > m_used + kRescaleLog2) {
          alpha = fast_exp2(m_used - m_tile);  // 0 when m_used = -inf
          m_used = m_tile;
        }
        const float nm = m_used == -INFINITY ? 0.0f : -m_used;
        float sum[8];
#pragma unroll
        for (int i8 = 0; i8 < 8; ++i8) sum[i8] = 0.0f;
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          fma2(s[c], s[c + 1], s[c], s[c + 1], sl2, sl2, nm, nm);
          if ((c & 15) == 14) {
            exp2_fma_pair(s[c], s[c + 1]);  // one pair in eight on the FMA pipe
          } else {
            s[c] = fast_exp2(s[c]);
            s[c + 1] = fast_exp2(s[c + 1]);
          }
          const int k = (c >> 1) & 3;  // four independent accumulator pairs
          add2(sum[2 * k], sum[2 * k + 1], sum[2 * k], sum[2 * k + 1], s[c], s[c + 1]);
          pk[c >> 1] = pack_bf16x2(s[c], s[c + 1]);
        }
        // keys [64 hf, +64) -> packed columns [32 hf, +32) of this buffer
        tmem_st32(scol + hf * 32, pk);
        l = l * alpha + (((sum[0] + sum[1]) + (sum[2] + sum[3])) + ((sum[4] + sum[5]) + (sum[6] + sum[7])));
        if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.0f)) {
          // O is quiescent once PV_{t-1} has completed (PV_t waits for this
          // P). Waited on only here: the issuer waited for PV_{t-3} before
          // S_t, and PV_{t+2} needs this warp's P, so the barrier of buffer
          // (t-1) % kSBufs is at PV_{t-1}'s phase or one past it.
          const int pb = (t - 1) % kSBufs;
          if (!warp_wait(&bars[kPVDone + pb], ((t - 1) / kSBufs) & 1)) {
            alive = false;
            break;
          }
          tc_fence_after();
          // this half rescales O columns [64 hf, +64)
          uint32_t o0[32], o1[32];
          const uint32_t oaddr = lane_base + kOCol + hf * 64;
          tmem_ld32(oaddr, o0);
          tmem_ld32(oaddr + 32, o1);
          tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            o0[c] = __float_as_uint(__uint_as_float(o0[c]) * alpha);
            o1[c] = __float_as_uint(__uint_as_float(o1[c]) * alpha);
          }
          tmem_st32(oaddr, o0);
          tmem_st32(oaddr + 32, o1);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        // One P barrier per S buffer: P_{t+3} needs S_{t+3}, hence PV_t, so
        // the issuer is never two phases behind it.
        if (lane == 0) mbar_arrive(&bars[kPFull + buf]);
      }
      if (!alive) break;
      // Row sum = both halves' sums; half 0 hands (max used, sum) to the
      // epilogue (one slot, freed by it).
      float lo;
      if (!exchange(l, lo)) break;
      if (hf == 0) {
        if (ix > 0 && !warp_wait(&bars[kStatsFree], (ix - 1) & 1)) break;
        // no finite score seen: the sum holds only clamped-exponent residue
        stats[r] = make_float2(m_used, m_used == -INFINITY ? 0.0f : l + lo);
        mbar_arrive(&bars[kStatsFull]);
      }
      ++ix;
    }
  } else {
    // ---------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem + (uint32_t(quad * 32) << 16);
    const int rq = r / p.group;
    int ix = 0;
    bool alive = true;
    Item it;
    for (int i = 0; alive && take_item(bars, ring, i, true, it); ++i) {
      const int qpos = it.q0 + rq;
      const bool valid_row = r < p.rows_used && rq < it.qx && qpos < p.max_q;
      const int head = it.h * p.group + (r - rq * p.group);
      __nv_bfloat16* dst = p.out + (((long long)it.q_begin + qpos) * p.qh + head) * 128;
      float* lse_dst = p.lse ? p.lse + ((long long)it.b * p.qh + head) * p.max_q + qpos : nullptr;
      if (it.n == 0) {
        // No visible keys (invalid context): zero rows, -inf LSE.
        if (valid_row) {
          for (int d = 0; d < 128; d += 8) *reinterpret_cast<uint4*>(dst + d) = make_uint4(0, 0, 0, 0);
          if (lse_dst) *lse_dst = -INFINITY;
        }
        continue;
      }
      if (!warp_wait(&bars[kStatsFull], ix & 1)) break;
      const float2 ml = stats[r];
      mbar_arrive(&bars[kStatsFree]);
      if (!warp_wait(&bars[kODone], ix & 1)) break;
      tc_fence_after();
      const float l = ml.y;
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t o0[32], o1[32];
        tmem_ld32(lane_base + kOCol + h * 64, o0);
        tmem_ld32(lane_base + kOCol + h * 64 + 32, o1);
        tmem_ld_wait();
        if (valid_row) {
#pragma unroll
          for (int vv = 0; vv < 8; ++vv) {
            const uint32_t* src = vv < 4 ? o0 + 8 * vv : o1 + 8 * (vv - 4);
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv);
            *reinterpret_cast<uint4*>(dst + h * 64 + vv * 8) = w;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kOFree]);
      if (valid_row && lse_dst) {
        const float m_out = ml.x == -INFINITY ? 0.0f : ml.x;
        *lse_dst = l > 0.0f ? (m_out + fast_log2(l)) * kLn2 : -INFINITY;
      }
      ++ix;
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
    if (atomicAdd(p.sched + 1, 1) == int(gridDim.x) - 1) {
      atomicExch(p.sched, 0);
      atomicExch(p.sched + 1, 0);
    }
  }
}

// Claim counters {next item, CTAs finished}, one pair per stream that
// launches the prefill (a launch leaves its pair at zero when it ends).
__device__ int g_prefill_tile_sched[64][2];

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
    *err = cudaGetSymbolAddress(&ptr, g_prefill_tile_sched);
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

}  // namespace prefill_tile_detail

cudaError_t launch_prefill_tile(const PrefillArgs& a, cudaStream_t stream) {
  using namespace prefill_tile_detail;
  const int group = a.qh / a.kvh;
  // Up to 128 query heads per kv head: a 128-row query tile holds 128 / group
  // queries of the group (at least one).
  if (group < 1 || group > kRows || a.batch > 65535 || a.kvh > 65535) return cudaErrorNotSupported;
  const int qt = kRows / group;
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
    return cudaFuncSetAttribute(prefill_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
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
  p.fd_nqt = FastDiv::make(p.n_qtiles > 0 ? p.n_qtiles : 1);
  p.fd_kvh = FastDiv::make(a.kvh);
  p.fd_qt = FastDiv::make(qt);
  p.fd_bs = FastDiv::make(a.block_size);
  const long long items = (long long)p.n_qtiles * a.batch * a.kvh;
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
  return cudaLaunchKernelEx(&cfg, prefill_tile_kernel, p, qmap, kmap, vmap);
}

}  // namespace nvb
