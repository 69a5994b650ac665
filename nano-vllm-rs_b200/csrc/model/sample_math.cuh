// Gumbel-max score arithmetic shared by the sampler (sample.cu) and the
// decode GEMM's sampling epilogue (gemm.cu), so both pick the same token from
// the same BF16 logits. The reference's stream and arithmetic
// (kernels/kernels.cu:371-377, 413-431): for temperature T > 0 and seed s,
// token v scores logit / T - logf(-logf(u)), u = ((x >> 41) + 0.5) / 2^23,
// x = SplitMix64(s ^ (v * 0xd2b74407b1ce6e93)); T == 0 scores the logit. The
// sample is the highest score, the lowest token index among equal scores.
#pragma once

#include <cstdint>

namespace nvbm {
namespace sample_math {

constexpr int kNone = 0x7fffffff;

__device__ __forceinline__ uint64_t splitmix64(uint64_t v) {
  v += 0x9e3779b97f4a7c15ULL;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ULL;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebULL;
  return v ^ (v >> 31);
}

// (score, index) is better than (best, best_index).
__device__ __forceinline__ bool better(float score, int index, float best, int best_index) {
  return score > best || (score == best && index < best_index);
}

__device__ __forceinline__ void warp_best(float& score, int& index) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float s = __shfl_xor_sync(0xffffffffu, score, off);
    const int i = __shfl_xor_sync(0xffffffffu, index, off);
    if (better(s, i, score, index)) {
      score = s;
      index = i;
    }
  }
}

__device__ __forceinline__ float gumbel_score(float logit, float temperature, uint64_t seed, int token) {
  if (!(temperature > 0.0f)) return logit;
  const uint64_t x = splitmix64(seed ^ (uint64_t(token) * 0xd2b74407b1ce6e93ULL));
  // x >> 41 has 23 bits: its 32-bit conversion is exact, like the 64-bit one.
  const float u = __fmul_rn(__fadd_rn(float(uint32_t(x >> 41)), 0.5f), 1.0f / 8388608.0f);
  return __fsub_rn(__fdiv_rn(logit, temperature), logf(-logf(u)));
}

}  // namespace sample_math
}  // namespace nvbm
