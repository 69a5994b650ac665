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
// One CTA handles one 128-row query tile of one (sequence, kv head). Rows pack
// the GQA group: row r = (query q0 + r / G, head h*G + r % G), so each K/V
// tile loaded from HBM serves all G query heads. Per 64-key KV tile j:
//
//   S_j = Q K_j^T   tcgen05.mma kind::f16, M=128 N=64 K=128 (8 x K16), A and
//                   B from 128B-swizzled shared memory, D in TMEM (FP32)
//   P_j = exp2(S_j * scale*log2e - m)   4 softmax warps, one TMEM lane (row)
//                   per thread, written back over S_j in TMEM as packed BF16
//   O  += P_j V_j   tcgen05.mma M=128 N=128 K=64 with A (P) read from TMEM,
//                   V as an MN-major B operand from shared memory, O in TMEM
//
// Warp roles: warp 0 issues TMA (Q once, then a 2-stage K ring and a 2-stage V
// ring over the sequence's pages: 3-D tensor maps over [tokens, kv_heads,
// 128] with 64-element, 128-byte-swizzled boxes; a 64-key tile never crosses
// a page since block_size is a multiple of 256); warp 1 owns TMEM (256
// columns: S double buffer at 0 and 64, O at 128) and one thread issues the
// MMAs and tcgen05.commit arrivals; warps 2..5 run the online softmax, the O
// rescale (TMEM ld/st) and the epilogue. S/P is double-buffered in TMEM and
// a buffer is released by the commit of the PV MMA that read its P; the
// softmax of tile j computes and stores P_j before it waits for PV_{j-1}.
//
// Sizing for B200: 96 KB of tiles + 1 KB of barriers per CTA and 256 TMEM
// columns let two CTAs share an SM (2 x 256 of the 512 columns), so one CTA's
// softmax runs while the other's MMAs use the tensor core, and their
// prologues/epilogues overlap. The softmax uses Blackwell's packed FP32x2
// FMA/ADD and three-input max to cut its instruction count, and evaluates an
// eighth of the exponentials on the FMA pipe (exp2_fma) next to the
// 16-per-clock MUFU unit.
//
// The kernel is persistent: 2 CTAs per SM loop over (query tile, sequence,
// kv head) items, longest causal tiles first, keeping their barriers and
// TMEM; the next item's Q load and first K/V tiles overlap the current
// item's last tiles and epilogue. Barrier phases are tracked with global
// tile and item counters; q_free (all S MMAs of an item done) and o_free (its
// epilogue has read O) guard the two buffers reused across items. The softmax keeps the
// running max it scales by unless a row's max grows by more than 2^8
// (FA4-style lazy rescale: P stays <= 256, exact after the final divide), so
// the TMEM read-modify-write of O is rare after the first tiles.
//
// Every wait is bounded (common.cuh); a timeout records an error code and the
// CTA still frees its TMEM and exits.
#include "internal.cuh"

namespace nvb {

namespace prefill_detail {

constexpr int kRows = 128;
constexpr int kKeys = 64;
constexpr int kStages = 2;
constexpr int kQHalf = kRows * 128;          // 128 rows x 64 BF16 (one 128-byte swizzle column)
constexpr int kQBytes = 2 * kQHalf;          // Q tile 128 x 128 BF16
constexpr int kKVHalf = kKeys * 128;         // 64 keys x 64 BF16
constexpr int kKVBytes = 2 * kKVHalf;        // K or V tile 64 x 128 BF16
constexpr int kThreads = 192;
constexpr int kTmemCols = 256;
constexpr int kOCol = 128;
constexpr float kLn2 = 0.693147180559945309f;
constexpr float kRescaleLog2 = 8.0f;         // lazy rescale threshold (P <= 2^8)

// Barriers and the TMEM slot sit below the first 1024-byte boundary; the
// tiles follow on 1024-byte boundaries (128-byte swizzle atoms).
enum Bar { kQFull = 0, kKFull = 1, kKEmpty = 3, kVFull = 5, kVEmpty = 7, kSFull = 9, kSFree = 11, kPFull = 13,
           kODone = 14, kQFree = 15, kOFree = 16, kNumBars = 17 };
constexpr int kTmemSlotOff = kNumBars * 8;
constexpr int kHeadBytes = kTmemSlotOff + 16;
constexpr int kQOff = 0;                      // offsets from the aligned tile base
constexpr int kKOff = kQOff + kQBytes;
constexpr int kVOff = kKOff + kStages * kKVBytes;
constexpr int kTileBytes = kVOff + kStages * kKVBytes;  // 96 KB
constexpr int kSmemBytes = 1024 + kTileBytes;           // 97 KB: two CTAs per SM

struct PrefillParams {
  int n_qtiles;  // query tiles of the longest sequence
  const int* cu_q;
  const int* kv_lens;
  const int* block_table;
  __nv_bfloat16* out;
  float* lse;
  int batch, max_q, qh, kvh, group, qt, rows_used, block_size, table_stride, num_blocks;
  float scale_log2;
};

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
// K-major, M = 128. S = Q K^T: B K-major, N = 64 keys. O += P V: B MN-major,
// N = 128 head dims.
constexpr uint32_t kIdescBase = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 4) << 24);
constexpr uint32_t kIdescS = kIdescBase | ((uint32_t(kKeys) >> 3) << 17);
constexpr uint32_t kIdescPV = kIdescBase | (1u << 16) | ((128u >> 3) << 17);

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// O += P V with A (P, packed BF16 pairs) read from tensor memory.
__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                                 uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// 2^x on the FMA/ALU pipes for x <= 128 (used for part of the softmax so the
// MUFU unit is not the limit). Range reduction x = n + f with n the nearest
// integer (1.5 * 2^23 rounding trick, |f| <= 1/2), then a degree-4
// polynomial for 2^f fitted to minimise relative error on [-1/2, 1/2] (this
// file's own fit; max relative error 2.7e-6 in FP32), then n is added to the
// exponent field. Inputs below -125 (masked keys are -inf) return exactly 0;
// the clamp keeps the exponent add from leaving the normal range.
__device__ __forceinline__ float exp2_fma(float x) {
  const float xc = fmaxf(x, -125.0f);
  const float t = xc + 12582912.0f;  // 1.5 * 2^23: low mantissa bits hold round(xc)
  const float f = xc - (t - 12582912.0f);
  float p = 0.009570096619427204f;
  p = fmaf(p, f, 0.05591785907745361f);
  p = fmaf(p, f, 0.240247443318367f);
  p = fmaf(p, f, 0.6931217908859253f);
  p = fmaf(p, f, 0.9999992847442627f);
  const float r = __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
  return x < -125.0f ? 0.0f : r;
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

// exp2_fma on a pair of inputs with the packed FP32 forms.
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
  const float ra = __int_as_float(__float_as_int(pa) + (__float_as_int(ta) << 23));
  const float rb = __int_as_float(__float_as_int(pb) + (__float_as_int(tb) << 23));
  a = a < -125.0f ? 0.0f : ra;
  b = b < -125.0f ? 0.0f : rb;
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

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %1, %1, %1};" ::"r"(addr), "r"(0) : "memory");
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ bool page_ok(int page, int num_blocks) { return page >= 0 && page < num_blocks; }

// One query tile of one (sequence, kv head): the work item of the
// persistent loop. Virtual items are ordered by query-tile index, longest
// causal tiles first, and dealt round-robin to the CTAs.
struct Item {
  int b, h, q_begin, q_len, q0, qt_eff, kv_len, prefix, key_end, n_tiles, full_tiles;
  bool empty;
};

__device__ __forceinline__ Item make_item(const PrefillParams& p, int v) {
  Item it;
  const int pairs = p.batch * p.kvh;
  const int tile = p.n_qtiles - 1 - v / pairs;
  const int rest = v % pairs;
  it.b = rest / p.kvh;
  it.h = rest % p.kvh;
  it.q_begin = p.cu_q[it.b];
  it.q_len = p.cu_q[it.b + 1] - it.q_begin;
  it.q0 = tile * p.qt;
  it.empty = it.q0 >= it.q_len;
  it.qt_eff = it.empty ? 0 : min(p.qt, it.q_len - it.q0);
  it.kv_len = it.empty ? 0 : p.kv_lens[it.b];
  it.prefix = it.kv_len - it.q_len;
  // A context longer than the page table, or shorter than its query group,
  // is invalid input: such rows get zero output (as decode does).
  const bool seq_ok = !it.empty && it.prefix >= 0 &&
                      (long long)it.kv_len <= (long long)p.table_stride * p.block_size;
  it.key_end = seq_ok ? min(it.kv_len, it.prefix + it.q0 + it.qt_eff) : 0;
  it.n_tiles = it.key_end > 0 ? (it.key_end + kKeys - 1) / kKeys : 0;
  const int free_keys = min(it.kv_len, it.prefix + it.q0 + 1);  // keys every row of the tile sees
  it.full_tiles = free_keys > 0 ? free_keys / kKeys : 0;
  return it;
}

__global__ void __launch_bounds__(kThreads, 2)
    prefill_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap qmap,
                   const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_addr(smem_raw);
  // tiles start at the first 1024-byte boundary past the barrier block
  const uint32_t tile_addr = (raw_addr + kHeadBytes + 1023u) & ~1023u;
  unsigned char* tiles = smem_raw + (tile_addr - raw_addr);
  const uint32_t sbase = tile_addr;
  if (tile_addr + kTileBytes > raw_addr + kSmemBytes) {  // dynamic smem base not 1 KB friendly
    if (threadIdx.x == 0) record_error(kErrPrefillAlign);
    return;
  }
  const int n_items = p.n_qtiles * p.batch * p.kvh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem_raw + kTmemSlotOff);
  if (threadIdx.x == 0) {
    mbar_init(&bars[kQFull], 1);
    mbar_init(&bars[kQFree], 1);
    mbar_init(&bars[kOFree], 4);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars[kKFull + s], 1);
      mbar_init(&bars[kKEmpty + s], 1);
      mbar_init(&bars[kVFull + s], 1);
      mbar_init(&bars[kVEmpty + s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kSFull + s], 1);
      mbar_init(&bars[kSFree + s], 1);
    }
    mbar_init(&bars[kPFull], 4);
    mbar_init(&bars[kODone], 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (warp >= 2 && p.rows_used < kRows) {
    // Rows past the packed (query, head) rows are never loaded: zero them once.
    const int t = threadIdx.x - 64;
    for (int e = t; e < (kRows - p.rows_used) * 16; e += 128) {
      const int r = p.rows_used + (e >> 4), c = e & 15;
      st_shared_zero16(sbase + kQOff + (c >> 3) * kQHalf + r * 128 + (c & 7) * 16);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // -------------------------------------------------------- TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      int gt = 0, it_count = 0;
      bool alive = true;
      for (int v = blockIdx.x; v < n_items && alive; v += gridDim.x) {
        const Item it = make_item(p, v);
        if (it.n_tiles == 0) continue;
        const int* table = p.block_table + (long long)it.b * p.table_stride;
        // Q of the previous item is free once all its S MMAs completed.
        if (it_count > 0 && !mbar_wait(&bars[kQFree], (it_count - 1) & 1, kErrPrefillWait)) break;
        mbar_arrive_expect_tx(&bars[kQFull], 2u * 128u * uint32_t(p.rows_used));
        const int qy = it.h * p.group, qz = it.q_begin + it.q0;
        tma_load_3d(tiles + kQOff, &qmap, &bars[kQFull], 0, qy, qz);
        tma_load_3d(tiles + kQOff + kQHalf, &qmap, &bars[kQFull], 64, qy, qz);
        for (int j = 0; j < it.n_tiles; ++j) {
          const int g = gt + j;
          const int st = g % kStages;
          const uint32_t par = ((g / kStages) + 1) & 1;
          const int key0 = j * kKeys;
          const int logical = key0 / p.block_size;
          const int page = table[logical];
          const bool ok = page_ok(page, p.num_blocks);
          const int trow = ok ? page * p.block_size + (key0 - logical * p.block_size) : 0;
          if (g >= kStages && !mbar_wait(&bars[kKEmpty + st], par, kErrPrefillWait)) { alive = false; break; }
          unsigned char* kdst = tiles + kKOff + st * kKVBytes;
          if (ok) {
            mbar_arrive_expect_tx(&bars[kKFull + st], kKVBytes);
            tma_load_3d(kdst, &kmap, &bars[kKFull + st], 0, it.h, trow);
            tma_load_3d(kdst + kKVHalf, &kmap, &bars[kKFull + st], 64, it.h, trow);
          } else {
            mbar_arrive(&bars[kKFull + st]);
          }
          if (g >= kStages && !mbar_wait(&bars[kVEmpty + st], par, kErrPrefillWait)) { alive = false; break; }
          unsigned char* vdst = tiles + kVOff + st * kKVBytes;
          if (ok) {
            mbar_arrive_expect_tx(&bars[kVFull + st], kKVBytes);
            tma_load_3d(vdst, &vmap, &bars[kVFull + st], 0, it.h, trow);
            tma_load_3d(vdst + kKVHalf, &vmap, &bars[kVFull + st], 64, it.h, trow);
          } else {
            mbar_arrive(&bars[kVFull + st]);
          }
        }
        gt += it.n_tiles;
        ++it_count;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t q_addr = sbase + kQOff;
      int gt = 0, it_count = 0;
      bool alive = true;
      // PV for global tile g; `first` starts a new item's accumulator, which
      // must wait until the previous item's epilogue has read O.
      auto issue_pv = [&](int g, bool first) {
        const int st = g % kStages;
        if (first && it_count > 0) alive = alive && mbar_wait(&bars[kOFree], (it_count - 1) & 1, kErrPrefillWait);
        alive = alive && mbar_wait(&bars[kPFull], g & 1, kErrPrefillWait);
        alive = alive && mbar_wait(&bars[kVFull + st], (g / kStages) & 1, kErrPrefillWait);
        if (!alive) return;
        tc_fence_after();
        const uint32_t v_addr = sbase + kVOff + st * kKVBytes;
        const uint32_t p_tmem = tmem + (g & 1) * kKeys;  // P_g over S_g: 16 keys = 8 columns
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint64_t bd = sw128_desc(v_addr + kk * 2048, kKVHalf, 1024);
          umma_bf16_tmem_a(tmem + kOCol, p_tmem + kk * 8, bd, kIdescPV, (!first || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bars[kVEmpty + st]);
        umma_commit(&bars[kODone]);
        umma_commit(&bars[kSFree + (g & 1)]);  // S/P buffer free once PV_g has read P_g
      };
      for (int v = blockIdx.x; v < n_items && alive; v += gridDim.x) {
        const Item it = make_item(p, v);
        if (it.n_tiles == 0) continue;
        alive = mbar_wait(&bars[kQFull], it_count & 1, kErrPrefillWait);
        tc_fence_after();
        for (int j = 0; j < it.n_tiles && alive; ++j) {
          const int g = gt + j;
          const int st = g % kStages, sb = g & 1;
          alive = mbar_wait(&bars[kKFull + st], (g / kStages) & 1, kErrPrefillWait);
          if (alive && g >= 2) alive = mbar_wait(&bars[kSFree + sb], ((g >> 1) + 1) & 1, kErrPrefillWait);
          if (!alive) break;
          tc_fence_after();
          const uint32_t k_addr = sbase + kKOff + st * kKVBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t qoff = (kk >> 2) * kQHalf + (kk & 3) * 32;
            const uint32_t koff = (kk >> 2) * kKVHalf + (kk & 3) * 32;
            umma_bf16(tmem + sb * kKeys, sw128_desc(q_addr + qoff, 16, 1024), sw128_desc(k_addr + koff, 16, 1024),
                      kIdescS, kk > 0 ? 1u : 0u);
          }
          umma_commit(&bars[kKEmpty + st]);
          umma_commit(&bars[kSFull + sb]);
          if (j >= 1) issue_pv(g - 1, j == 1);
        }
        if (!alive) break;
        umma_commit(&bars[kQFree]);  // every S MMA of this item has been issued
        issue_pv(gt + it.n_tiles - 1, it.n_tiles == 1);
        gt += it.n_tiles;
        ++it_count;
      }
    }
  } else {
    // ---------------------------------------------- softmax and epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // TMEM lane = packed row
    const uint32_t trow = tmem + (uint32_t(quad * 32) << 16);
    const int rq = r / p.group;
    const float sl2 = p.scale_log2;
    int gt = 0;
    bool alive = true;
    for (int v = blockIdx.x; v < n_items && alive; v += gridDim.x) {
      const Item it = make_item(p, v);
      if (it.empty) continue;
      const int head = it.h * p.group + (r % p.group);
      const bool valid_row = r < p.rows_used && rq < it.qt_eff;
      const long long tok = (long long)it.q_begin + it.q0 + rq;
      if (it.n_tiles == 0) {
        // No visible keys (invalid context): zero rows, -inf LSE.
        if (valid_row) {
          __nv_bfloat16* dst = p.out + (tok * p.qh + head) * 128;
          for (int d = 0; d < 128; d += 8) *reinterpret_cast<uint4*>(dst + d) = make_uint4(0, 0, 0, 0);
          if (p.lse) p.lse[((long long)it.b * p.qh + head) * p.max_q + it.q0 + rq] = -INFINITY;
        }
        continue;
      }
      const int* table = p.block_table + (long long)it.b * p.table_stride;
      const int limit = valid_row ? it.prefix + it.q0 + rq : it.key_end - 1;  // last visible key
      float m_used = -INFINITY, l = 0.0f;  // running max the probabilities are scaled by
      for (int j = 0; j < it.n_tiles; ++j) {
        const int g = gt + j;
        const int sb = g & 1;
        const int key0 = j * kKeys;
        const bool ok = page_ok(table[key0 / p.block_size], p.num_blocks);
        if (!mbar_wait(&bars[kSFull + sb], (g >> 1) & 1, kErrPrefillWait)) {
          alive = false;
          break;
        }
        tc_fence_after();
        float s[kKeys];
        {
          uint32_t raw0[32], raw1[32];
          tmem_ld32(trow + sb * kKeys, raw0);
          tmem_ld32(trow + sb * kKeys + 32, raw1);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            s[i] = __uint_as_float(raw0[i]);
            s[32 + i] = __uint_as_float(raw1[i]);
          }
        }
        if (j >= it.full_tiles || !ok) {
          const int lim = ok ? min(limit, it.kv_len - 1) - key0 : -1;
#pragma unroll
          for (int c = 0; c < kKeys; ++c)
            if (c > lim) s[c] = -INFINITY;
        }
        float mx8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx8[i] = s[i];
#pragma unroll
        for (int c = 8; c < kKeys; c += 16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) mx8[i] = max3(mx8[i], s[c + i], s[c + 8 + i]);
        }
        const float mx = max3(max3(mx8[0], mx8[1], mx8[2]), max3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
        const float m_tile = mx * sl2;
        // Rescale only when the row max grew by more than 2^8 (or on the
        // first finite max); otherwise keep scaling by the stale max.
        float alpha = 1.0f;
        if (m_tile > m_used + kRescaleLog2) {
          alpha = fast_exp2(m_used - m_tile);  // 0 when m_used = -inf
          m_used = m_tile;
        }
        const float nm = m_used == -INFINITY ? 0.0f : -m_used;
        float sum[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) sum[i] = 0.0f;
#pragma unroll
        for (int c = 0; c < kKeys; c += 2) {
          fma2(s[c], s[c + 1], s[c], s[c + 1], sl2, sl2, nm, nm);
          if ((c & 15) == 14) {
            exp2_fma_pair(s[c], s[c + 1]);  // one pair in eight on the FMA pipe
          } else {
            s[c] = fast_exp2(s[c]);
            s[c + 1] = fast_exp2(s[c + 1]);
          }
          const int k = (c >> 1) & 3;  // four independent accumulator pairs
          add2(sum[2 * k], sum[2 * k + 1], sum[2 * k], sum[2 * k + 1], s[c], s[c + 1]);
        }
        l = l * alpha + (((sum[0] + sum[1]) + (sum[2] + sum[3])) + ((sum[4] + sum[5]) + (sum[6] + sum[7])));

        // P_g as packed BF16 pairs over the first 32 columns of S_g.
        {
          uint32_t pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = pack_bf16x2(s[2 * i], s[2 * i + 1]);
          tmem_st32(trow + sb * kKeys, pk);
        }
        // One o_done phase per tile (PV_{g-1}); the item's first tile needs
        // none: the previous epilogue consumed that phase.
        if (j >= 1) {
          if (!mbar_wait(&bars[kODone], (g - 1) & 1, kErrPrefillWait)) {
            alive = false;
            break;
          }
          tc_fence_after();
        }
        // V rows that are not real keys (past kv_len, or an invalid page) are
        // zeroed so that P = 0 never meets a non-finite cache value. All PVs
        // before g are complete here, so this vfull wait is for V_g itself.
        const int real_keys = ok ? min(kKeys, it.kv_len - key0) : 0;
        if (real_keys < kKeys) {
          const int st = g % kStages;
          if (!mbar_wait(&bars[kVFull + st], (g / kStages) & 1, kErrPrefillWait)) {
            alive = false;
            break;
          }
          if (r < kKeys && r >= real_keys) {
            const uint32_t vrow = sbase + kVOff + st * kKVBytes + r * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              st_shared_zero16(vrow + c * 16);
              st_shared_zero16(vrow + kKVHalf + c * 16);
            }
          }
          fence_proxy_async_smem();
        }
        if (j >= 1 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t o0[32], o1[32];
            const uint32_t oaddr = trow + kOCol + half * 64;
            tmem_ld32(oaddr, o0);
            tmem_ld32(oaddr + 32, o1);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              o0[i] = __float_as_uint(__uint_as_float(o0[i]) * alpha);
              o1[i] = __float_as_uint(__uint_as_float(o1[i]) * alpha);
            }
            tmem_st32(oaddr, o0);
            tmem_st32(oaddr + 32, o1);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars[kPFull]);
      }
      if (!alive) break;

      // epilogue: O / l -> BF16 rows of `out`, natural-log LSE; then O is free
      const int g_last = gt + it.n_tiles - 1;
      if (!mbar_wait(&bars[kODone], g_last & 1, kErrPrefillWait)) break;
      tc_fence_after();
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      __nv_bfloat16* dst = p.out + (tok * p.qh + head) * 128;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t o0[32], o1[32];
        tmem_ld32(trow + kOCol + half * 64, o0);
        tmem_ld32(trow + kOCol + half * 64 + 32, o1);
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
            *reinterpret_cast<uint4*>(dst + half * 64 + vv * 8) = w;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kOFree]);
      if (valid_row && p.lse) {
        const float m_out = m_used == -INFINITY ? 0.0f : m_used;
        p.lse[((long long)it.b * p.qh + head) * p.max_q + it.q0 + rq] =
            l > 0.0f ? (m_out + fast_log2(l)) * kLn2 : -INFINITY;
      }
      gt += it.n_tiles;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace prefill_detail

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream) {
  using namespace prefill_detail;
  const int group = a.qh / a.kvh;
  if (group < 1 || group > 16 || a.batch > 65535 || a.kvh > 65535) return cudaErrorNotSupported;
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

  const CUtensorMap *qmap = nullptr, *kmap = nullptr, *vmap = nullptr;
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
  static unsigned long long configured = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(__atomic_load_n(&configured, __ATOMIC_ACQUIRE) & bit)) {
    e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return e;
    __atomic_fetch_or(&configured, bit, __ATOMIC_RELEASE);
  }
  static int sm_count[64] = {};
  if (!sm_count[dev & 63]) {
    int n = 0;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sm_count[dev & 63] = n;
  }
  p.n_qtiles = (a.max_q + qt - 1) / qt;
  const long long items = (long long)p.n_qtiles * a.batch * a.kvh;
  if (items > 0x7fffffffLL) return cudaErrorNotSupported;
  const int grid = int(items < 2LL * sm_count[dev & 63] ? items : 2LL * sm_count[dev & 63]);
  prefill_kernel<<<grid, kThreads, kSmemBytes, stream>>>(p, *qmap, *kmap, *vmap);
  return cudaGetLastError();
}

}  // namespace nvb
