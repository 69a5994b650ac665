// Gumbel-max sampling over BF16 logits (libnvb_model.so).
//
// Token parity with the reference engine needs the reference's random
// stream and score arithmetic exactly (kernels/kernels.cu:371-377, 413-431):
// for row r with temperature T > 0 and seed s, token v scores
//   logit / T - logf(-logf(u)),  u = ((x >> 41) + 0.5) / 2^23,
//   x = SplitMix64(s ^ (v * 0xd2b74407b1ce6e93)),
// and T == 0 scores the logit itself. The sample is the highest score, the
// lowest token index among equal scores, and token 0 when no score is
// comparable (all NaN). That choice is a lexicographic maximum, so it does
// not depend on how the vocabulary is cut into partitions or on the order
// partial results are merged; the partition layout here is this library's.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "model_internal.cuh"
#include "sample_math.cuh"

namespace nvbm {

namespace {

using namespace sample_math;

constexpr int kThreads = 256;
constexpr int kPerThread = 16;
constexpr int kPartition = kThreads * kPerThread;  // tokens per CTA

// grid (partitions, rows): the best (score, index) of one partition of a row.
__global__ void sample_partition_kernel(const __nv_bfloat16* __restrict__ logits, const float* __restrict__ temps,
                                        const uint64_t* __restrict__ seeds, float* __restrict__ part_score,
                                        int* __restrict__ part_index, int vocab) {
  const int part = blockIdx.x, row = blockIdx.y, parts = gridDim.x;
  const float temperature = temps[row];
  const uint64_t seed = seeds[row];
  const __nv_bfloat16* in = logits + (long long)row * vocab;
  float best = -INFINITY;
  int best_index = kNone;
  const int begin = part * kPartition;
#pragma unroll 4
  for (int e = 0; e < kPerThread; ++e) {
    const int token = begin + e * kThreads + int(threadIdx.x);  // increasing per thread
    if (token < vocab) {
      const float score = gumbel_score(__bfloat162float(in[token]), temperature, seed, token);
      if (better(score, token, best, best_index)) {
        best = score;
        best_index = token;
      }
    }
  }
  warp_best(best, best_index);
  __shared__ float s_score[kThreads / 32];
  __shared__ int s_index[kThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_score[warp] = best;
    s_index[warp] = best_index;
  }
  __syncthreads();
  if (warp == 0) {
    best = lane < kThreads / 32 ? s_score[lane] : -INFINITY;
    best_index = lane < kThreads / 32 ? s_index[lane] : kNone;
    warp_best(best, best_index);
    if (lane == 0) {
      part_score[(long long)row * parts + part] = best;
      part_index[(long long)row * parts + part] = best_index;
    }
  }
}

// One warp per row folds the partition results.
__global__ void sample_combine_kernel(const float* __restrict__ part_score, const int* __restrict__ part_index,
                                      int* __restrict__ out, int rows, int parts) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float best = -INFINITY;
  int best_index = kNone;
  for (int p = lane; p < parts; p += 32) {
    const float s = part_score[(long long)row * parts + p];
    const int i = part_index[(long long)row * parts + p];
    if (better(s, i, best, best_index)) {
      best = s;
      best_index = i;
    }
  }
  warp_best(best, best_index);
  if (lane == 0) out[row] = best_index == kNone ? 0 : best_index;
}

}  // namespace

int sample_partitions(int vocab) { return (vocab + kPartition - 1) / kPartition; }

cudaError_t launch_sample(cudaStream_t s, const void* logits, const float* temps, const uint64_t* seeds, int* out,
                          float* part_score, int* part_index, int rows, int vocab) {
  const int parts = sample_partitions(vocab);
  if (rows <= 0 || rows > 65535) return cudaErrorInvalidValue;
  sample_partition_kernel<<<dim3(parts, rows), kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(logits), temps,
                                                                 seeds, part_score, part_index, vocab);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  sample_combine_kernel<<<(rows + 3) / 4, 128, 0, s>>>(part_score, part_index, out, rows, parts);
  return cudaGetLastError();
}

cudaError_t launch_sample_combine(cudaStream_t s, const float* part_score, const int* part_index, int* out, int rows,
                                  int parts) {
  if (rows <= 0 || parts <= 0) return cudaErrorInvalidValue;
  sample_combine_kernel<<<(rows + 3) / 4, 128, 0, s>>>(part_score, part_index, out, rows, parts);
  return cudaGetLastError();
}

}  // namespace nvbm
