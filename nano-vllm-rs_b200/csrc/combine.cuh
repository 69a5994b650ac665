// Split-KV combine of one (row, q head) item, shared by combine_kernel
// (decode.cu) and the fused combine + all-gather (gather.cu), so both give the
// same bits. Each split s left a normalised partial row O_s and its LSE; the
// item's output is sum_s w_s O_s / sum_s w_s with w_s = exp(lse_s - max lse)
// (kernels/decode_candidate.cuh:180-201 restated in LSE form).
//
// The sum over splits is latency-bound when there are many splits and few
// items (long contexts on few sequences: 74 splits of 4 rows x 8 heads at
// the config-5 shard of 8 GPUs), so W warps share an item, each takes a
// contiguous range of splits and loads eight splits' LSEs and partial rows
// before it adds any, and the W shares are added in warp order. The order of
// every addition depends only on the split count: the result is
// deterministic, and with W = 1 it is the plain split-order sum.
#pragma once

#include "common.cuh"

namespace nvb {
namespace combine_detail {

constexpr int kCombineThreads = 256;  // 8 warps
constexpr int kCombineBatch = 8;      // splits whose loads a warp issues before adding

// Warps sharing one item: the smallest power of two (at most 8) for which no
// warp takes more than one batch of splits.
inline int combine_warps(int splits) {
  int w = 1;
  while (w < 8 && w * kCombineBatch < splits) w <<= 1;
  return w;
}

// Share `sub` (of W) of item `item`: acc (this lane's 4 dims of sum w_s O_s
// over the share's splits), total (sum w_s), mx (max lse over all splits, the
// same in every share; -inf when no split saw a key).
template <int W>
__device__ __forceinline__ void combine_share(const float* __restrict__ lse_accum, const float* __restrict__ out_accum,
                                              long long item, long long stride, int splits, int sub, int lane,
                                              float4& acc, float& total, float& mx) {
  mx = -INFINITY;
  for (int s = lane; s < splits; s += 32) mx = fmaxf(mx, lse_accum[s * stride + item]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  acc = make_float4(0.f, 0.f, 0.f, 0.f);
  total = 0.0f;
  if (mx == -INFINITY) return;
  const int per = (splits + W - 1) / W;
  const int s0 = sub * per, s1 = min(splits, s0 + per);
  for (int base = s0; base < s1; base += kCombineBatch) {
    float ls[kCombineBatch];
    float4 v[kCombineBatch];
#pragma unroll
    for (int u = 0; u < kCombineBatch; ++u) {
      const int s = base + u;
      if (s < s1) {
        ls[u] = lse_accum[s * stride + item];
        v[u] = *reinterpret_cast<const float4*>(out_accum + (s * stride + item) * 128 + lane * 4);
      }
    }
#pragma unroll
    for (int u = 0; u < kCombineBatch; ++u) {
      if (base + u >= s1 || ls[u] == -INFINITY) continue;
      const float w = __expf(ls[u] - mx);
      total += w;
      acc.x = fmaf(w, v[u].x, acc.x);
      acc.y = fmaf(w, v[u].y, acc.y);
      acc.z = fmaf(w, v[u].z, acc.z);
      acc.w = fmaf(w, v[u].w, acc.w);
    }
  }
}

// Adds the other W - 1 shares of this warp's item (the warps right after it)
// to the first share, in warp order. Every thread of the CTA calls it.
template <int W>
__device__ __forceinline__ void combine_gather_shares(float4& acc, float& total, int warp, int lane, int sub) {
  __shared__ float4 s_acc[kCombineThreads / 32][32];
  __shared__ float s_tot[kCombineThreads / 32];
  if (W > 1) {
    s_acc[warp][lane] = acc;
    if (lane == 0) s_tot[warp] = total;
    __syncthreads();
    if (sub == 0) {
#pragma unroll
      for (int w = 1; w < W; ++w) {
        const float4 o = s_acc[warp + w][lane];
        acc.x += o.x;
        acc.y += o.y;
        acc.z += o.z;
        acc.w += o.w;
        total += s_tot[warp + w];
      }
    }
  }
}

}  // namespace combine_detail
}  // namespace nvb
