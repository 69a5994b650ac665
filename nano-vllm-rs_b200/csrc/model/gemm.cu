// Decode-shaped GEMMs on tcgen05 tensor cores (sm_100a): Y[M, N] = X[M, K] W[N, K]^T
// for the few rows of a decode step (M <= 256), BF16 in and out, FP32
// accumulation. Replaces the cublasGemmEx call of the reference's forward
// (kernels/kernels.cu:98-106) for those shapes; prefill-sized GEMMs stay on
// cuBLAS.
//
// A decode step's GEMMs stream weights: at M = 256 a layer of Qwen3-0.6B reads
// 30 MB of weights against 8 GFLOP, and the library GEMMs ran at 4-8 us per
// launch. Here the roles are swapped so that the weights are the MMA's M:
//
//   D^T[128 features, M] += W_tile[128 features, 64 k] X_tile[M, 64 k]^T
//   A = W tile (K-major, 128B-swizzled, TMA), B = X tile (K-major, TMA; rows
//   past M are TMA zero fill), D in TMEM (lane = feature, column = row).
//
// A CTA owns 128 output features (or, for the fused SiLU epilogue, 64 gate
// features and the 64 matching up features, so each output's gate and up sit
// in one CTA) and a slice of K. The S CTAs that split one tile's K form a
// thread-block cluster (co-scheduled, so they may wait on one another): each
// stores its FP32 partial [M][128] into a caller-provided workspace that
// stays in L2, and after a cluster barrier CTA r sums rows
// [r*M/S, (r+1)*M/S) of the S partials, always in rank order (deterministic:
// a CUDA-graph replay gives the eager result bit for bit), and writes BF16
// outputs. No atomics. (Moving the partials through distributed shared
// memory instead was measured 3-7x slower: 85-115 KB per CTA at M = 256.)
//
// Warp roles: warp 0 TMA producer, warp 1 TMEM owner and MMA issuer, warps
// 2..5 move the accumulator out of TMEM; all six warps sum and store.
// Waits are bounded (about two seconds) and record an error word that
// nvbe_gemm_device_error() reads, so a fault in the pipeline surfaces as an
// error instead of a hung GPU.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "model_internal.cuh"
#include "sample_math.cuh"

namespace nvbm {

namespace gemm_detail {

constexpr int kThreads = 192;
constexpr int kBK = 64;                    // k per stage: one 128-byte row per operand row
constexpr int kTileN = 128;                // features per CTA (MMA M)
constexpr int kWBytes = kTileN * kBK * 2;  // 16 KB
constexpr int kDataBytes = 192 * 1024;     // stage ring; the epilogue's receive buffer reuses it
constexpr int kMaxStages = 8;
constexpr int kMaxCluster = 16;
constexpr int kHeadBytes = 1024;           // barriers, TMEM address
constexpr int kSmemBytes = kHeadBytes + kDataBytes + 1024;  // + 1 KB to align the ring
constexpr long long kWaitCycles = 4000000000LL;

__device__ int g_gemm_error = 0;

struct Params {
  int M, N, K;        // X [M, K], W [N, K]; silu: N = 2 * inter
  int mpad;           // M rounded up to 16 (the MMA's N)
  int kb_total;       // K / 64
  int cluster;        // CTAs splitting one tile's K
  int stages;
  int silu;           // 0: Y[M, N]; 1: Y[M, N / 2] = silu(gate) * up
  int sample;         // 1: Y = BF16 logits, plus each row's best Gumbel-max (score, token) per tile
  float* ws;          // FP32 partials [tiles][cluster][M][128] (L2-resident scratch)
  const float* temps;       // sample: [M] temperatures
  const uint64_t* seeds;    // sample: [M] seeds
  float* part_score;        // sample: [M][tiles]
  int* part_index;          // sample: [M][tiles]
  int tiles;
  __nv_bfloat16* y;
  int ldy;            // elements per output row
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const long long start = clock64();
  while (!mbar_try(bar, parity)) {
    if (clock64() - start > kWaitCycles) {
      atomicCAS(&g_gemm_error, 0, 1);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand, 128-byte swizzle: 128-byte rows, 8-row groups 1 KB apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(16 >> 4) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// kind::f16, FP32 accumulate, BF16 A and B, both K-major, M = 128, N = n.
__device__ __forceinline__ uint32_t idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t(n) >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(id), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// The reference's SiLU * up on BF16 gate and up values (kernels/kernels.cu:
// 355-364, the same arithmetic as silu_mul_kernel in layers.cu).
__device__ __forceinline__ float silu_mul(float g, float u) {
  const float gate = __bfloat162float(__float2bfloat16_rn(g));
  const float up = __bfloat162float(__float2bfloat16_rn(u));
  const float activation = __fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate)));
  return __fmul_rn(activation, up);
}

enum { kBarFull = 0, kBarEmpty = kMaxStages, kBarDone = 2 * kMaxStages, kNumBars };
constexpr int kTmemSlot = kNumBars * 8;
constexpr int kSampleOff = 512;  // sampling epilogue: float [16][4] scores, int [16][4] tokens
static_assert(kTmemSlot + 4 <= kSampleOff && kSampleOff + 16 * 4 * 8 <= kHeadBytes, "head layout overlaps");

// kMode: 0 plain, 1 SiLU * up, 2 sampling (one instantiation each, so the
// sampling epilogue carries no split-K registers and two of its CTAs share an
// SM, overlapping one CTA's epilogue with the other's weight stream).
template <int kMode>
__global__ void __launch_bounds__(kThreads, kMode == 2 ? 2 : 1)
    gemm_decode_kernel(const Params p, const __grid_constant__ CUtensorMap wmap,
                       const __grid_constant__ CUtensorMap xmap) {
  // Launched as a programmatic dependent of the kernel before it: the next
  // kernel may be scheduled now, and everything below that reads the input
  // rows or writes memory waits (griddepcontrol.wait) for the previous
  // kernel to complete. The weights do not depend on it: their first stages
  // load before the wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t ring = (raw + kHeadBytes + 1023u) & ~1023u;
  const uint32_t bars = raw;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = int(cluster_rank());
  const int tile = blockIdx.x / p.cluster;
  const int stage_bytes = kWBytes + p.mpad * 128;
  // This CTA's k blocks: the first (kb_total % cluster) ranks take one more.
  const int kb_base = p.kb_total / p.cluster, kb_extra = p.kb_total % p.cluster;
  const int kb0 = rank * kb_base + min(rank, kb_extra);
  const int nkb = kb_base + (rank < kb_extra ? 1 : 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(bars + 8 * (kBarFull + s), 1);
      mbar_init(bars + 8 * (kBarEmpty + s), 1);
    }
    mbar_init(bars + 8 * kBarDone, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  uint32_t tmem_cols = 32;
  while (tmem_cols < uint32_t(p.mpad)) tmem_cols <<= 1;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(raw + kTmemSlot),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem_raw + kTmemSlot);

  // This CTA's FP32 partial [M][128] in the workspace: slot (tile, rank).
  float* part = kMode == 2 ? nullptr : p.ws + ((long long)tile * p.cluster + rank) * p.M * kTileN;
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && nkb > 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&wmap)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
      auto load_w = [&](int i) {
        const int s = i % p.stages;
        const uint32_t full = bars + 8 * (kBarFull + s);
        const uint32_t dst = ring + s * stage_bytes;
        const int k = (kb0 + i) * kBK;
        mbar_expect_tx(full, uint32_t(stage_bytes));  // W and X bytes of the stage
        if (kMode == 1) {
          const int inter = p.N / 2, f0 = tile * (kTileN / 2);
          tma_load_2d(dst, &wmap, full, k, f0);                        // gate rows -> tile rows 0..63
          tma_load_2d(dst + kWBytes / 2, &wmap, full, k, inter + f0);  // up rows -> tile rows 64..127
        } else {
          tma_load_2d(dst, &wmap, full, k, tile * kTileN);
        }
      };
      auto load_x = [&](int i) {
        const int s = i % p.stages;
        tma_load_2d(ring + s * stage_bytes + kWBytes, &xmap, bars + 8 * (kBarFull + s), (kb0 + i) * kBK, 0);
      };
      const int early = nkb < p.stages ? nkb : p.stages;
      for (int i = 0; i < early; ++i) load_w(i);
      asm volatile("griddepcontrol.wait;" ::: "memory");  // the input rows are written
      for (int i = 0; i < early; ++i) load_x(i);
      for (int i = early; i < nkb; ++i) {
        const int s = i % p.stages;
        if (!mbar_wait(bars + 8 * (kBarEmpty + s), ((i / p.stages) + 1) & 1)) break;
        load_w(i);
        load_x(i);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id = idesc(p.mpad);
      bool alive = true;
      for (int i = 0; i < nkb && alive; ++i) {
        const int s = i % p.stages;
        alive = mbar_wait(bars + 8 * (kBarFull + s), (i / p.stages) & 1);
        if (!alive) break;
        tc_fence_after();
        const uint32_t a = ring + s * stage_bytes, b = a + kWBytes;
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          umma(tmem, sw128_desc(a + kk * 32), sw128_desc(b + kk * 32), id, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(bars + 8 * (kBarEmpty + s));
      }
      // Done: every MMA above has completed (or none ran: nkb == 0).
      if (nkb > 0) umma_commit(bars + 8 * kBarDone);
      else asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bars + 8 * kBarDone) : "memory");
    }
  } else {
    // ------------------------------------- TMEM -> this CTA's workspace slot
    // One 128-byte store per warp and row (lane = feature); the slots stay
    // in L2 for the sum below.
    const int quad = warp & 3;
    const int f = quad * 32 + lane;  // feature row of the tile (TMEM lane)
    asm volatile("griddepcontrol.wait;" ::: "memory");  // before any global write
    const bool done = __all_sync(0xffffffffu, mbar_wait(bars + 8 * kBarDone, 0));
    tc_fence_after();
    const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16);
    if constexpr (kMode == 2) {
      // Logits of 128 tokens for every row: rounded to BF16 as the plain
      // GEMM rounds them (stored, for the caller's diagnostics), scored with
      // the sampler's Gumbel arithmetic, and folded to this tile's best
      // (score, token) per row: warps, then the four warps through shared
      // memory (named barrier 1 over the 128 epilogue threads).
      using namespace sample_math;
      float* slot_score = reinterpret_cast<float*>(smem_raw + kSampleOff);  // [16 rows][4 warps]
      int* slot_index = reinterpret_cast<int*>(smem_raw + kSampleOff + 16 * 4 * 4);
      const int n = tile * kTileN + f;
      const int t = (warp - 2) * 32 + lane;
      for (int c = 0; c < p.M; c += 16) {
        uint32_t r[16];
        if (done && nkb > 0) {
          tmem_ld16(taddr + uint32_t(c), r);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) r[j] = 0u;
        }
        // The chunk's 16 scores first (independent: their latencies
        // overlap), then the 16 warp folds.
        float score[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = c + j;
          score[j] = -INFINITY;
          if (m < p.M && n < p.N) {
            const __nv_bfloat16 lb = __float2bfloat16_rn(__uint_as_float(r[j]));
            p.y[(long long)m * p.ldy + n] = lb;
            score[j] = gumbel_score(__bfloat162float(lb), p.temps[m], p.seeds[m], n);
          }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (c + j >= p.M) break;
          float sc = score[j];
          int index = n < p.N ? n : kNone;
          warp_best(sc, index);
          if (lane == 0) {
            slot_score[j * 4 + quad] = sc;
            slot_index[j * 4 + quad] = index;
          }
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (t < 16 && c + t < p.M) {
          float best = slot_score[t * 4];
          int best_index = slot_index[t * 4];
          for (int q = 1; q < 4; ++q)
            if (better(slot_score[t * 4 + q], slot_index[t * 4 + q], best, best_index)) {
              best = slot_score[t * 4 + q];
              best_index = slot_index[t * 4 + q];
            }
          p.part_score[(long long)(c + t) * p.tiles + tile] = best;
          p.part_index[(long long)(c + t) * p.tiles + tile] = best_index;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
      }
    }
    for (int c = 0; c < p.M && done && kMode != 2; c += 16) {
      uint32_t r[16];
      if (nkb > 0) {
        tmem_ld16(taddr + uint32_t(c), r);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) r[j] = 0u;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (c + j < p.M) __stcg(part + (long long)(c + j) * kTileN + f, __uint_as_float(r[j]));
    }
    tc_fence_before();
  }

  // Every partial of the cluster is in the workspace (release / acquire at
  // cluster scope orders the global stores before the loads below).
  cluster_sync();

  // ------------------------------------------ sum in rank order, epilogue
  // CTA r of the cluster owns rows [r*rows_per, ...); item (row, 4 features),
  // consecutive threads on consecutive features.
  const int rows_per = (p.M + p.cluster - 1) / p.cluster;
  const int m0 = rank * rows_per, rows = max(0, min(p.M, m0 + rows_per) - m0);
  const float* base = p.ws + (long long)tile * p.cluster * p.M * kTileN;
  const long long slot = (long long)p.M * kTileN;
  if constexpr (kMode == 2) {
    // done in the epilogue above
  } else if constexpr (kMode == 0) {
    const int n0 = tile * kTileN;
    for (int e = threadIdx.x; e < rows * (kTileN / 4); e += kThreads) {
      const int m = m0 + e / (kTileN / 4), c4 = (e % (kTileN / 4)) * 4;
      if (n0 + c4 >= p.N) continue;
      const float* src = base + (long long)m * kTileN + c4;
      // All S partials are loaded before the first add (one L2 latency per
      // output, not S), then summed in rank order.
      float4 v[kMaxCluster];
#pragma unroll
      for (int s = 0; s < kMaxCluster; ++s)
        if (s < p.cluster) v[s] = __ldcg(reinterpret_cast<const float4*>(src + s * slot));
      float4 acc = v[0];
#pragma unroll
      for (int s = 1; s < kMaxCluster; ++s) {
        if (s >= p.cluster) break;
        acc.x += v[s].x;
        acc.y += v[s].y;
        acc.z += v[s].z;
        acc.w += v[s].w;
      }
      uint2 out;
      out.x = pack2(acc.x, acc.y);
      out.y = pack2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(p.y + (long long)m * p.ldy + n0 + c4) = out;
    }
  } else {
    const int inter = p.N / 2, i0 = tile * (kTileN / 2);
    for (int e = threadIdx.x; e < rows * (kTileN / 8); e += kThreads) {
      const int m = m0 + e / (kTileN / 8), c4 = (e % (kTileN / 8)) * 4;
      if (i0 + c4 >= inter) continue;
      const float* src = base + (long long)m * kTileN + c4;
      float4 gv[kMaxCluster], uv[kMaxCluster];
#pragma unroll
      for (int s = 0; s < kMaxCluster; ++s)
        if (s < p.cluster) {
          gv[s] = __ldcg(reinterpret_cast<const float4*>(src + s * slot));
          uv[s] = __ldcg(reinterpret_cast<const float4*>(src + s * slot + kTileN / 2));
        }
      float4 g = gv[0], u = uv[0];
#pragma unroll
      for (int s = 1; s < kMaxCluster; ++s) {
        if (s >= p.cluster) break;
        g.x += gv[s].x;
        g.y += gv[s].y;
        g.z += gv[s].z;
        g.w += gv[s].w;
        u.x += uv[s].x;
        u.y += uv[s].y;
        u.z += uv[s].z;
        u.w += uv[s].w;
      }
      uint2 out;
      out.x = pack2(silu_mul(g.x, u.x), silu_mul(g.y, u.y));
      out.y = pack2(silu_mul(g.z, u.z), silu_mul(g.w, u.w));
      *reinterpret_cast<uint2*>(p.y + (long long)m * p.ldy + i0 + c4) = out;
    }
  }

  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
  }
}

}  // namespace gemm_detail

int gemm_decode_max_rows() { return 256; }

// Measured against cublasGemmEx in CUDA graphs on B200 (Qwen3-0.6B shapes,
// weights streamed from HBM): this kernel is faster up to 8 rows for every
// projection (the 4096-output QKV projection drew level at 16), and up to 64
// rows for outputs of at most 2048 features (few tiles, so K splits over
// large clusters); past that the split-K partials, which grow with the rows,
// cost more than cuBLAS's whole GEMM.
bool gemm_decode_preferred(int M, int N, int K) {
  (void)K;
  return M >= 1 && (M <= 8 || (N <= 2048 && M <= 64));
}

// The LM head with the sampler fused (measured the same way against
// cublasGemmEx + the sampler, vocabulary 151936): faster at one row (63.5
// vs 68.5 us), even at 8, slower from 16 (the per-row scoring epilogue).
bool gemm_sample_preferred(int M) { return M >= 1 && M <= 4; }

namespace {

// The kernel's shared-memory size and cluster-size attributes, once per
// device (before any launch or occupancy query).
cudaError_t configure_kernel() {
  using namespace gemm_detail;
  static std::mutex mu;
  static int configured_device = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (configured_device == dev) return cudaSuccess;
  for (auto fn : {gemm_decode_kernel<0>, gemm_decode_kernel<1>, gemm_decode_kernel<2>}) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  }
  if (e == cudaSuccess) configured_device = dev;
  return e;
}

// Clusters of `size` CTAs of the decode GEMM that fit the device at once,
// cached per (device, size); 0 when it cannot be determined.
int max_clusters(int size) {
  if (configure_kernel() != cudaSuccess) return 0;
  static std::mutex mu;
  static int cache_dev = -1;
  static int cache[17] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cache_dev != dev) {
    for (int& c : cache) c = -1;
    cache_dev = dev;
  }
  if (cache[size] < 0) {
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(size);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(unsigned(size));
    cfg.blockDim = dim3(gemm_detail::kThreads);
    cfg.dynamicSmemBytes = gemm_detail::kSmemBytes;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    cache[size] = cudaOccupancyMaxActiveClusters(&n, gemm_detail::gemm_decode_kernel<0>, &cfg) == cudaSuccess ? n : 0;
  }
  return cache[size];
}

}  // namespace

int gemm_decode_cluster(int M, int N, int K, bool silu, int sms) {
  using namespace gemm_detail;
  const int features = silu ? N / 2 : N, per_tile = silu ? kTileN / 2 : kTileN;
  const int tiles = (features + per_tile - 1) / per_tile, kb_total = K / kBK;
  // The most K slices (at most 16, at least two k blocks each) whose grid
  // still fits one CTA per SM and whose clusters are all resident at once.
  // A grid whose clusters do not all fit at once runs a second wave (measured:
  // 48 clusters of 3 started up to 6 us late), so the occupancy check applies
  // to every size.
  (void)M;
  for (int c = kMaxCluster; c > 1; --c) {
    if (tiles * c > sms || kb_total / c < 2) continue;
    if (max_clusters(c) < tiles) continue;
    return c;
  }
  return 1;
}

size_t gemm_decode_workspace(int M, int N, int K, bool silu, int sms) {
  using namespace gemm_detail;
  if (M < 1 || N < 1 || K < kBK) return 0;
  const int features = silu ? N / 2 : N, per_tile = silu ? kTileN / 2 : kTileN;
  const size_t tiles = size_t((features + per_tile - 1) / per_tile);
  return tiles * size_t(gemm_decode_cluster(M, N, K, silu, sms)) * size_t(M) * kTileN * sizeof(float);
}

int gemm_decode_tiles(int N) { return (N + gemm_detail::kTileN - 1) / gemm_detail::kTileN; }

namespace {
cudaError_t launch_impl(cudaStream_t stream, const CUtensorMap& wmap, const CUtensorMap& xmap, gemm_detail::Params p,
                        int tiles);
}  // namespace

cudaError_t launch_gemm_decode_sample(cudaStream_t stream, const CUtensorMap& wmap, const CUtensorMap& xmap,
                                      void* logits, int M, int N, int K, const float* temps, const uint64_t* seeds,
                                      float* part_score, int* part_index) {
  using namespace gemm_detail;
  if (M < 1 || M > 256 || N < 4 || N % 4 || K < kBK || K % kBK || !logits || !temps || !seeds || !part_score ||
      !part_index || (reinterpret_cast<uintptr_t>(logits) & 7))
    return cudaErrorInvalidValue;
  if (cudaError_t e = configure_kernel(); e != cudaSuccess) return e;
  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.mpad = (M + 15) / 16 * 16;
  p.kb_total = K / kBK;
  p.sample = 1;
  p.y = static_cast<__nv_bfloat16*>(logits);
  p.ldy = N;
  // Four stages: at most 16 rows that is 72 KB, so two CTAs share an SM
  // (three, with three stages, measured no faster).
  p.stages = kDataBytes / (kWBytes + p.mpad * 128);
  if (p.stages > 4) p.stages = 4;
  p.cluster = 1;  // each CTA holds whole logits for its tokens
  p.temps = temps;
  p.seeds = seeds;
  p.part_score = part_score;
  p.part_index = part_index;
  p.tiles = gemm_decode_tiles(N);
  return launch_impl(stream, wmap, xmap, p, p.tiles);
}

cudaError_t launch_gemm_decode(cudaStream_t stream, const CUtensorMap& wmap, const CUtensorMap& xmap, void* y,
                               int M, int N, int K, int ldy, bool silu, int sms, void* ws, size_t ws_bytes) {
  using namespace gemm_detail;
  if (M < 1 || M > 256 || N < 4 || N % 4 || K < kBK || K % kBK || (silu && N % 8) || ldy < 1 || ldy % 4 ||
      (reinterpret_cast<uintptr_t>(y) & 7))
    return cudaErrorInvalidValue;
  if (cudaError_t e = configure_kernel(); e != cudaSuccess) return e;
  Params p{};
  p.M = M;
  p.N = N;
  p.K = K;
  p.mpad = (M + 15) / 16 * 16;
  p.kb_total = K / kBK;
  p.silu = silu ? 1 : 0;
  p.y = static_cast<__nv_bfloat16*>(y);
  p.ldy = ldy;
  const int stage_bytes = kWBytes + p.mpad * 128;
  p.stages = kDataBytes / stage_bytes;
  if (p.stages > kMaxStages) p.stages = kMaxStages;
  const int features = silu ? N / 2 : N;
  const int per_tile = silu ? kTileN / 2 : kTileN;
  const int tiles = (features + per_tile - 1) / per_tile;
  if (reinterpret_cast<uintptr_t>(ws) & 15) return cudaErrorInvalidValue;
  // Cluster size: the most K slices (at most 16, at least two k blocks each)
  // whose grid still fits one CTA per SM; past the portable 8 only when that
  // many clusters of the size can be resident at once.
  const int cluster = gemm_decode_cluster(M, N, K, silu, sms);
  p.cluster = cluster;
  if (!ws || ws_bytes < gemm_decode_workspace(M, N, K, silu, sms)) return cudaErrorInvalidValue;
  p.ws = static_cast<float*>(ws);
  return launch_impl(stream, wmap, xmap, p, tiles);
}

namespace {
cudaError_t launch_impl(cudaStream_t stream, const CUtensorMap& wmap, const CUtensorMap& xmap, gemm_detail::Params p,
                        int tiles) {
  using namespace gemm_detail;
  const int cluster = p.cluster;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(tiles * cluster));
  cfg.blockDim = dim3(kThreads);
  // The ring holds p.stages stages; the split-K forms also reuse it for
  // their receive space, so they take the whole budget.
  cfg.dynamicSmemBytes = p.sample ? kHeadBytes + 1024 + p.stages * (kWBytes + p.mpad * 128) : kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (p.sample) return cudaLaunchKernelEx(&cfg, gemm_decode_kernel<2>, p, wmap, xmap);
  if (p.silu) return cudaLaunchKernelEx(&cfg, gemm_decode_kernel<1>, p, wmap, xmap);
  return cudaLaunchKernelEx(&cfg, gemm_decode_kernel<0>, p, wmap, xmap);
}
}  // namespace

int encode_map_2d(const void* base, uint64_t inner, uint64_t rows, uint32_t box_inner, uint32_t box_rows,
                  CUtensorMap* out) {
  using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(ptr);
  });
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (inner * 2) % 16) return -1;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner * 2};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  return fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? 0
             : -1;
}

int gemm_weight_map(const void* w, int N, int K, bool silu, CUtensorMap* out) {
  return encode_map_2d(w, uint64_t(K), uint64_t(N), 64, silu ? 64 : 128, out);
}

int gemm_input_map(const void* x, int M, int K, CUtensorMap* out) {
  return encode_map_2d(x, uint64_t(K), uint64_t(M), 64, uint32_t((M + 15) / 16 * 16), out);
}

int gemm_decode_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gemm_detail::g_gemm_error, sizeof(int)) != cudaSuccess) return -1;
  return v;
}

}  // namespace nvbm
