// Split-KV paged decode attention for B200 (sm_100a).
//
// Replaces the reference's decode paths: the native ordered kernel
// (kernels/kernels.cu:288-354, one CTA per (row, q head), K/V re-read once per
// query head) and the FA2 split-KV decode behind nvr_flash_fwd
// (kernels/flash_native/flash_native.cu:61-112). Math follows the split-KV
// partial / combine algorithm of kernels/decode_candidate.cuh:111-202
// (partial = normalised O plus its log-sum-exp; combine weights each split
// by exp(lse_s - max lse)).
//
// Design (decode is HBM-bound, ~2-8 FLOP per byte):
//  * One CTA per (query row, kv head, head group, split). The whole GQA query
//    group of that kv head shares every K/V tile read from HBM.
//  * Warp 0 is a TMA producer: a 3-D tensor map over the cache
//    [tokens = num_blocks * block_size, kv_heads, 128] loads 32-token K and V
//    tiles (8 KB each, box {128, 1, 32}) of the sequence's pages into a
//    6-stage shared-memory ring. A 32-token tile never crosses a page
//    because block_size is a multiple of 32.
//  * Warps 1..4 are consumers; consumer w owns tiles w, w+4, ... and keeps
//    its own online-softmax state (m, l, O). Each lane owns 8 of the 128
//    head dimensions (one 16-byte shared-memory load per K/V row); the two
//    half-warps take alternate tokens. QK partial sums are reduced with a
//    transpose-reduce shuffle (each step halves the values a lane holds), so
//    a 16-token dot product costs ~1 shuffle per token instead of 4.
//  * Phase tracking: mbarrier parity waits are only sound when a waiter is
//    never two phases behind or ahead of its barrier. With 6 stages shared
//    round-robin by 4 warps a warp meets a given stage only every other use,
//    so each stage has two "full" barriers, one for its even and one for its
//    odd uses. Use k-2 of a stage is tile i-12, which belongs to the same
//    warp (12 = 0 mod 4), so each warp waits on every phase of the barriers
//    it uses, in order. The producer waits on every phase of the "empty"
//    barriers.
//  * At the end the four warp states merge through shared memory, and the
//    CTA writes the final BF16 output (1 split) or a normalised FP32 partial
//    plus its natural-log LSE (several splits) for the combine kernel.
#include "internal.cuh"
#include "combine.cuh"

namespace nvb {

namespace decode_detail {

constexpr int kTile = kDecodeTile;  // tokens per pipeline stage
constexpr int kStages = 6;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = 32 * (1 + kConsumerWarps);
constexpr int kRowBytes = 256;
constexpr int kTileBytes = kTile * kRowBytes;
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kMaxPageCache = 256;
constexpr float kLn2 = 0.693147180559945309f;

template <int GC>
struct Smem {
  static constexpr int kStageOff = 0;
  static constexpr int kPOff = kStages * kStageBytes;                        // P scratch per warp
  static constexpr int kPBytes = kConsumerWarps * GC * kTile * 4;
  static constexpr int kBarOff = kPOff + kPBytes;                            // full[], empty[]
  static constexpr int kPageOff = kBarOff + 3 * kStages * 8;  // full[2 * kStages], empty[kStages]
  static constexpr int kValidOff = kPageOff + kMaxPageCache * 4;
  static constexpr int kBytes = kValidOff + kStages * 4;
  // Merge area reuses the stage ring after the pipeline has drained.
  static constexpr int kMergeBytes = kConsumerWarps * GC * (2 + 128) * 4;
  static_assert(kMergeBytes <= kStages * kStageBytes, "merge area must fit in the stage ring");
  static_assert((2 * kStages) % kConsumerWarps == 0,
                "uses k and k-2 of a stage must belong to the same consumer warp");
};

template <int GC>
__device__ __forceinline__ void write_empty(const DecodeParams& p, int row, int head0, int split,
                                            long long lse_base) {
  // Rows with no keys: zero output and -inf LSE (the reference writes zeros
  // for invalid rows, kernels/kernels.cu:294-297), or an empty split partial
  // (O = 0, lse = -inf) that the combine kernel ignores.
  for (int e = threadIdx.x; e < GC * 128; e += blockDim.x) {
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
}

template <int GC>
__global__ void __launch_bounds__(kThreads) decode_kernel(const DecodeParams p,
                                                          const __grid_constant__ CUtensorMap kmap,
                                                          const __grid_constant__ CUtensorMap vmap) {
  using S = Smem<GC>;
  constexpr int kHalfTok = kTile / 2;          // tokens per half-warp per tile
  constexpr int kTok = GC <= 4 ? 16 : 8;       // tokens per half-warp per pass
  constexpr int kPasses = kHalfTok / kTok;
  constexpr int kShift = kTok == 16 ? 0 : 1;   // after the reduce, lane s holds token s >> kShift
  extern __shared__ __align__(1024) unsigned char smem[];

  int cta = blockIdx.x;
  const int split = cta % p.num_splits;
  cta /= p.num_splits;
  const int hgroup = cta % p.n_hgroups;
  cta /= p.n_hgroups;
  const int kvhead = cta % p.kvh;
  const int row = cta / p.kvh;
  const int group = p.qh / p.kvh;
  const int head0 = kvhead * group + hgroup * GC;

  // Sequence metadata. Native mode mirrors kernels/kernels.cu:292-297;
  // varlen mode applies the bottom-right causal rule of
  // kernels/flash_native/flash_native.cu:102-104 (query i of a q_len-query
  // group sees kv_len - q_len + i + 1 keys).
  int seq, len, qi = 0;
  bool valid;
  if (p.mode == kModeNative) {
    seq = p.seq_map[row];
    const long long ctx = (long long)p.lens[row] + 1;
    valid = seq >= 0 && seq < p.batch && ctx >= 1 && ctx <= p.max_context &&
            ctx <= (long long)p.table_stride * p.block_size;
    len = valid ? int(ctx) : 0;
  } else if (p.mode == kModeVarlen) {
    int lo = 0, hi = p.batch - 1;  // last b with cu_q[b] <= row
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.seq_map[mid] <= row) lo = mid; else hi = mid - 1;
    }
    seq = lo;
    const int qlen = p.seq_map[seq + 1] - p.seq_map[seq];
    qi = row - p.seq_map[seq];
    const long long ctx = (long long)p.lens[seq] - qlen + qi + 1;
    valid = qi >= 0 && qi < qlen && ctx >= 1 && ctx <= (long long)p.table_stride * p.block_size;
    len = valid ? int(ctx) : 0;
  } else {
    seq = row;
    len = p.lens[row];
    valid = len >= 1 && (long long)len <= (long long)p.table_stride * p.block_size;
  }
  const long long lse_base = ((long long)seq * p.qh) * p.max_q + qi;
  const int n_tiles_total = valid ? (len + kTile - 1) / kTile : 0;
  const int per_split = (n_tiles_total + p.num_splits - 1) / p.num_splits;
  const int t0 = split * per_split;
  const int t1 = min(t0 + per_split, n_tiles_total);
  const int ntiles = max(0, t1 - t0);
  if (ntiles == 0) {
    write_empty<GC>(p, row, head0, split, lse_base);
    return;
  }

  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* empty = full + 2 * kStages;  // full[2 * stage + (use & 1)]
  int* pages = reinterpret_cast<int*>(smem + S::kPageOff);
  int* stage_valid = reinterpret_cast<int*>(smem + S::kValidOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int* table = p.block_table + (long long)seq * p.table_stride;
  const int first_page = (t0 * kTile) / p.block_size;
  const int n_pages = ((t1 * kTile - 1) / p.block_size) - first_page + 1;
  const bool cache_pages = n_pages <= kMaxPageCache;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[2 * s], 1);
      mbar_init(&full[2 * s + 1], 1);
      mbar_init(&empty[s], 1);
    }
    fence_barrier_init();
  }
  if (warp == 0 && cache_pages) {
    for (int i = lane; i < n_pages; i += 32) pages[i] = table[first_page + i];
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      const uint64_t policy = policy_evict_first();
      for (int i = 0; i < ntiles; ++i) {
        const int stage = i % kStages;
        if (i >= kStages) {
          if (!mbar_wait(&empty[stage], ((i / kStages) + 1) & 1, kErrDecodeEmptyWait)) break;
        }
        const int token0 = (t0 + i) * kTile;
        const int logical = token0 / p.block_size;
        const int offset = token0 - logical * p.block_size;
        const int page = cache_pages ? pages[logical - first_page] : table[logical];
        const bool ok = page >= 0 && page < p.num_blocks;
        uint64_t* fb = &full[2 * stage + ((i / kStages) & 1)];
        stage_valid[stage] = ok ? 1 : 0;
        if (ok) {
          unsigned char* kdst = smem + S::kStageOff + stage * kStageBytes;
          const int trow = page * p.block_size + offset;
          mbar_arrive_expect_tx(fb, kStageBytes);
          tma_load_3d_hint(kdst, &kmap, fb, 0, kvhead, trow, policy);
          tma_load_3d_hint(kdst + kTileBytes, &vmap, fb, 0, kvhead, trow, policy);
        } else {
          mbar_arrive(fb);
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int cw = warp - 1;
  const int h = lane >> 4, s = lane & 15;
  float qf[GC][8];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p.q + ((long long)row * p.qh + head0 + g) * 128 + s * 8);
    unpack8(raw, qf[g]);
#pragma unroll
    for (int d = 0; d < 8; ++d) qf[g][d] *= p.scale_log2;
  }
  float m[GC], l[GC], o[GC][8];
#pragma unroll
  for (int g = 0; g < GC; ++g) {
    m[g] = -INFINITY;
    l[g] = 0.0f;
#pragma unroll
    for (int d = 0; d < 8; ++d) o[g][d] = 0.0f;
  }
  float* P = reinterpret_cast<float*>(smem + S::kPOff) + cw * GC * kTile;  // [g][h][kHalfTok]
  const bool dup_writer = (s & ((1 << kShift) - 1)) == 0;

  for (int i = cw; i < ntiles; i += kConsumerWarps) {
    const int stage = i % kStages;
    const int use = i / kStages;
    if (!mbar_wait(&full[2 * stage + (use & 1)], (use >> 1) & 1, kErrDecodeFullWait)) break;
    const bool ok = stage_valid[stage] != 0;
    const int ntok = min(kTile, len - (t0 + i) * kTile);
    const unsigned char* kt = smem + S::kStageOff + stage * kStageBytes;
    const unsigned char* vt = kt + kTileBytes;

    // ---- scores: sc[pass][g] for token pass*2*kTok + 2*(s >> kShift) + h
    float sc[kPasses][GC];
#pragma unroll
    for (int pp = 0; pp < kPasses; ++pp) {
      float part[GC][kTok];
#pragma unroll
      for (int j = 0; j < kTok; ++j) {
        const int token = pp * 2 * kTok + 2 * j + h;
        const uint4 raw = *reinterpret_cast<const uint4*>(kt + token * kRowBytes + s * 16);
        float kf[8];
        unpack8(raw, kf);
#pragma unroll
        for (int g = 0; g < GC; ++g) {
          float acc = qf[g][0] * kf[0];
#pragma unroll
          for (int d = 1; d < 8; ++d) acc = fmaf(qf[g][d], kf[d], acc);
          part[g][j] = acc;
        }
      }
      // transpose-reduce across the 16 lanes of each half-warp
#pragma unroll
      for (int g = 0; g < GC; ++g) {
        int n = kTok;
#pragma unroll
        for (int mask = 8; mask >= 1; mask >>= 1) {
          if (n > 1) {
            const bool upper = (s & mask) != 0;
#pragma unroll
            for (int j = 0; j < kTok / 2; ++j) {
              if (j < n / 2) {
                const float keep = upper ? part[g][j + n / 2] : part[g][j];
                const float send = upper ? part[g][j] : part[g][j + n / 2];
                part[g][j] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
              }
            }
            n >>= 1;
          } else {
            part[g][0] += __shfl_xor_sync(0xffffffffu, part[g][0], mask);
          }
        }
        const int token = pp * 2 * kTok + 2 * (s >> kShift) + h;
        sc[pp][g] = (ok && token < ntok) ? part[g][0] : -INFINITY;
      }
    }

    // ---- online softmax update (log2 domain)
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      float mt = sc[0][g];
#pragma unroll
      for (int pp = 1; pp < kPasses; ++pp) mt = fmaxf(mt, sc[pp][g]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_new = fmaxf(m[g], mt);
      float alpha = 1.0f;
      if (m_new != -INFINITY) {
        alpha = fast_exp2(m[g] - m_new);
        m[g] = m_new;
      }
      l[g] *= alpha;
#pragma unroll
      for (int d = 0; d < 8; ++d) o[g][d] *= alpha;
#pragma unroll
      for (int pp = 0; pp < kPasses; ++pp) {
        const float pr = (sc[pp][g] == -INFINITY) ? 0.0f : fast_exp2(sc[pp][g] - m_new);
        if (dup_writer) {
          l[g] += pr;
          P[g * kTile + h * kHalfTok + pp * kTok + (s >> kShift)] = pr;
        }
      }
    }
    __syncwarp();

    // ---- O += P V over this half-warp's 16 tokens
    if (ok) {
      const float* Ph = P + h * kHalfTok;
      if (ntok == kTile) {
#pragma unroll
        for (int j4 = 0; j4 < kHalfTok; j4 += 4) {
          float4 pr[GC];
#pragma unroll
          for (int g = 0; g < GC; ++g) pr[g] = *reinterpret_cast<const float4*>(Ph + g * kTile + j4);
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            const int token = 2 * (j4 + jj) + h;
            const uint4 raw = *reinterpret_cast<const uint4*>(vt + token * kRowBytes + s * 16);
            float vf[8];
            unpack8(raw, vf);
#pragma unroll
            for (int g = 0; g < GC; ++g) {
              const float w = jj == 0 ? pr[g].x : jj == 1 ? pr[g].y : jj == 2 ? pr[g].z : pr[g].w;
#pragma unroll
              for (int d = 0; d < 8; ++d) o[g][d] = fmaf(w, vf[d], o[g][d]);
            }
          }
        }
      } else {
        const int cnt = (ntok - h + 1) >> 1;  // tokens 2j + h < ntok
        for (int j = 0; j < cnt; ++j) {
          const int token = 2 * j + h;
          const uint4 raw = *reinterpret_cast<const uint4*>(vt + token * kRowBytes + s * 16);
          float vf[8];
          unpack8(raw, vf);
#pragma unroll
          for (int g = 0; g < GC; ++g) {
            const float w = Ph[g * kTile + j];
#pragma unroll
            for (int d = 0; d < 8; ++d) o[g][d] = fmaf(w, vf[d], o[g][d]);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
  }

  // ---- merge the two half-warps, then the consumer warps
#pragma unroll
  for (int g = 0; g < GC; ++g) {
#pragma unroll
    for (int d = 0; d < 8; ++d) o[g][d] += __shfl_xor_sync(0xffffffffu, o[g][d], 16);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) l[g] += __shfl_xor_sync(0xffffffffu, l[g], off);
  }
  // All K/V tiles of this CTA have been consumed; the ring is free for reuse.
  named_barrier(1, kConsumerWarps * 32);
  float* Mw = reinterpret_cast<float*>(smem);          // [warp][g]
  float* Lw = Mw + kConsumerWarps * GC;                 // [warp][g]
  float* Ow = Lw + kConsumerWarps * GC;                 // [warp][g][128]
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      Mw[cw * GC + g] = m[g];
      Lw[cw * GC + g] = l[g];
    }
  }
  if (h == 0) {
#pragma unroll
    for (int g = 0; g < GC; ++g) {
      float4* dst = reinterpret_cast<float4*>(Ow + (cw * GC + g) * 128 + s * 8);
      dst[0] = make_float4(o[g][0], o[g][1], o[g][2], o[g][3]);
      dst[1] = make_float4(o[g][4], o[g][5], o[g][6], o[g][7]);
    }
  }
  named_barrier(1, kConsumerWarps * 32);
  const int ct = threadIdx.x - 32;
  for (int e = ct; e < GC * 128; e += kConsumerWarps * 32) {
    const int g = e >> 7, d = e & 127;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, Mw[w * GC + g]);
    float L = 0.0f, acc = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float mw = Mw[w * GC + g];
        const float sw = mw == -INFINITY ? 0.0f : fast_exp2(mw - M);
        L += Lw[w * GC + g] * sw;
        acc += Ow[(w * GC + g) * 128 + d] * sw;
      }
    }
    const int head = head0 + g;
    const float lse = L > 0.0f ? (M + fast_log2(L)) * kLn2 : -INFINITY;
    const float val = L > 0.0f ? acc / L : 0.0f;
    if (p.num_splits == 1) {
      p.out[((long long)row * p.qh + head) * 128 + d] = __float2bfloat16_rn(val);
      if (d == 0 && p.lse) p.lse[lse_base + (long long)head * p.max_q] = lse;
    } else {
      p.out_accum[(((long long)split * p.rows + row) * p.qh + head) * 128 + d] = val;
      if (d == 0) p.lse_accum[((long long)split * p.rows + row) * p.qh + head] = lse;
    }
  }
}

// W warps per (row, q head) item (combine.cuh): each split's normalised
// partial weighted by exp(lse_s - max_s lse_s) (kernels/decode_candidate.cuh:
// 180-201 restated in LSE form); BF16 output plus the final LSE.
template <int W>
__global__ void __launch_bounds__(combine_detail::kCombineThreads)
    combine_kernel(const float* __restrict__ lse_accum, const float* __restrict__ out_accum,
                   __nv_bfloat16* __restrict__ out, float* __restrict__ lse, int rows, int qh, int splits,
                   int lse_stride) {
  // Launched as a programmatic dependent of the decode grid: wait until that
  // grid has completed and its partials are visible (a no-op otherwise).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = warp % W;
  const long long item = (long long)blockIdx.x * (combine_detail::kCombineThreads / 32 / W) + warp / W;
  const bool live = item < (long long)rows * qh;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float total = 0.0f, mx = -INFINITY;
  if (live)
    combine_detail::combine_share<W>(lse_accum, out_accum, item, (long long)rows * qh, splits, sub, lane, acc, total,
                                     mx);
  combine_detail::combine_gather_shares<W>(acc, total, warp, lane, sub);
  if (!live || sub != 0) return;
  const float inv = total > 0.0f ? 1.0f / total : 0.0f;
  uint2 packed;
  packed.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  packed.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(out + item * 128 + lane * 4) = packed;
  if (lane == 0 && lse) lse[item * lse_stride] = total > 0.0f ? mx + __logf(total) : -INFINITY;
}

template <int GC>
cudaError_t launch_gc(const DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      cudaStream_t stream) {
  constexpr int bytes = Smem<GC>::kBytes;
  // The dynamic shared-memory opt-in belongs to the context; set it once per context.
  static unsigned configured[kContextSlots] = {};
  cudaError_t e = once_per_context(configured, [] {
    return cudaFuncSetAttribute(decode_kernel<GC>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  if (e != cudaSuccess) return e;
  const long long grid = (long long)p.rows * p.kvh * p.n_hgroups * p.num_splits;
  if (grid <= 0 || grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  decode_kernel<GC><<<unsigned(grid), kThreads, bytes, stream>>>(p, kmap, vmap);
  return cudaGetLastError();
}

}  // namespace decode_detail

int decode_group_chunk(int group) {
  using namespace decode_detail;
  // Heads of one GQA group processed by one CTA: the largest divisor <= 8.
  for (int gc = 8; gc >= 1; --gc)
    if (group % gc == 0) return gc;
  return 1;
}

cudaError_t launch_decode(DecodeParams p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                          cudaStream_t stream) {
  using namespace decode_detail;
  const int group = p.qh / p.kvh;
  const int gc = decode_group_chunk(group);
  p.n_hgroups = group / gc;
  cudaError_t e;
  switch (gc) {
    case 1: e = launch_gc<1>(p, kmap, vmap, stream); break;
    case 2: e = launch_gc<2>(p, kmap, vmap, stream); break;
    case 3: e = launch_gc<3>(p, kmap, vmap, stream); break;
    case 4: e = launch_gc<4>(p, kmap, vmap, stream); break;
    case 5: e = launch_gc<5>(p, kmap, vmap, stream); break;
    case 6: e = launch_gc<6>(p, kmap, vmap, stream); break;
    case 7: e = launch_gc<7>(p, kmap, vmap, stream); break;
    default: e = launch_gc<8>(p, kmap, vmap, stream); break;
  }
  if (e != cudaSuccess || p.num_splits == 1) return e;
  return launch_combine(p, stream);
}

cudaError_t launch_combine(const DecodeParams& p, cudaStream_t stream) {
  using namespace decode_detail;
  const long long items = (long long)p.rows * p.qh;
  const int w = combine_detail::combine_warps(p.num_splits);
  const int per_cta = combine_detail::kCombineThreads / 32 / w;  // items a CTA combines
  const long long grid = (items + per_cta - 1) / per_cta;
  // Programmatic stream serialization: the combine's launch overlaps the
  // decode grid's tail instead of following its completion.
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(combine_detail::kCombineThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const float* la = static_cast<const float*>(p.lse_accum);
  const float* oa = static_cast<const float*>(p.out_accum);
  switch (w) {
    case 1: return cudaLaunchKernelEx(&cfg, combine_kernel<1>, la, oa, p.out, p.lse, p.rows, p.qh, p.num_splits, p.max_q);
    case 2: return cudaLaunchKernelEx(&cfg, combine_kernel<2>, la, oa, p.out, p.lse, p.rows, p.qh, p.num_splits, p.max_q);
    case 4: return cudaLaunchKernelEx(&cfg, combine_kernel<4>, la, oa, p.out, p.lse, p.rows, p.qh, p.num_splits, p.max_q);
    default:
      return cudaLaunchKernelEx(&cfg, combine_kernel<8>, la, oa, p.out, p.lse, p.rows, p.qh, p.num_splits, p.max_q);
  }
}

}  // namespace nvb
