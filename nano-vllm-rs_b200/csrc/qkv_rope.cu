// Fused per-head Q/K RMSNorm + rotate-half RoPE + paged KV store (sm_100a).
//
// Follows the arithmetic of the reference's qkv_rope_kernel
// (kernels/kernels.cu:166-211) so results are bit-identical, but is laid out
// for B200: one warp per (row, head) instead of one 256-thread CTA, so a
// 148-SM part runs thousands of heads per wave and no CTA-wide barrier is
// needed.
//
// Bit-exactness argument. The reference's block_sum (kernels.cu:113-125)
// sums the 128 squared elements with thread j holding element j: warp w
// reduces elements [32w, 32w+32) with a shfl_down tree, then lanes 0..7 of
// warp 0 reduce the 8 warp partials (4..7 are zero) with the same tree,
// which evaluates to (P0 + P2) + (P1 + P3). Here lane l holds elements
// l, l+32, l+64, l+96, runs the same shfl_down tree on each of the four
// registers (giving P0..P3 at lane 0), and forms (P0 + P2) + (P1 + P3).
// Adding the reference's zero partials is exact, so the FP32 sum, the
// rsqrtf, the BF16 rounding of the normalised value (kernels.cu:185) and the
// non-contracted RoPE products (kernels.cu:203-204) all match.
#include "internal.cuh"

namespace nvb {

namespace rope_detail {

__device__ __forceinline__ float tree_sum_down(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
  return v;
}

template <bool CACHED>
__global__ void __launch_bounds__(256) qkv_rope_kernel(
    const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ qweight,
    const __nv_bfloat16* __restrict__ kweight, const int* __restrict__ positions,
    const int* __restrict__ slots, __nv_bfloat16* __restrict__ qout, __nv_bfloat16* __restrict__ kcache,
    __nv_bfloat16* __restrict__ vcache, int rows, int qheads, int kvheads, int block_size,
    int num_blocks, float eps, float theta, const float* __restrict__ rope_cache, int max_positions) {
  // The decode launched after this kernel as a programmatic dependent may be
  // scheduled now (its set-up overlaps this grid); it waits for this grid to
  // complete before it reads the new tokens.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  constexpr int kDim = 128, kHalf = 64;
  const int lane = threadIdx.x & 31;
  const int heads = qheads + kvheads;
  const long long item = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= (long long)rows * heads) return;
  const int row = int(item / heads), head = int(item % heads);
  const bool is_q = head < qheads;
  const int local_head = is_q ? head : head - qheads;
  const long long packed = (long long)row * (qheads + 2 * kvheads) * kDim;
  const __nv_bfloat16* x = qkv + packed + (long long)head * kDim;
  const __nv_bfloat16* w = is_q ? qweight : kweight;

  float v[4], sq[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[i] = __bfloat162float(x[lane + 32 * i]);
    sq[i] = v[i] * v[i];
  }
  float part[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) part[i] = tree_sum_down(sq[i]);
  float total = (part[0] + part[2]) + (part[1] + part[3]);
  total = __shfl_sync(0xffffffffu, total, 0);
  const float inv_rms = rsqrtf(total / kDim + eps);

  float n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float norm = v[i] * inv_rms;
    n[i] = __bfloat162float(__float2bfloat16_rn(norm * __bfloat162float(w[lane + 32 * i])));
  }

  const int position = positions[row];
  const int slot = slots[row];
  float cosv[2], sinv[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int pair = lane + 32 * i;  // elements j and j + 64 share a pair
    if constexpr (CACHED) {
      const bool valid = position >= 0 && position < max_positions;
      cosv[i] = valid ? rope_cache[(long long)position * kDim + pair] : 1.0f;
      sinv[i] = valid ? rope_cache[(long long)position * kDim + kHalf + pair] : 0.0f;
    } else {
      const float angle = position * powf(theta, -float(2 * pair) / kDim);
      sincosf(angle, &sinv[i], &cosv[i]);
    }
  }
  float r[4];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    r[i] = __fsub_rn(__fmul_rn(n[i], cosv[i]), __fmul_rn(n[i + 2], sinv[i]));
    r[i + 2] = __fadd_rn(__fmul_rn(n[i + 2], cosv[i]), __fmul_rn(n[i], sinv[i]));
  }

  if (is_q) {
    __nv_bfloat16* dst = qout + ((long long)row * qheads + local_head) * kDim;
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = __float2bfloat16_rn(r[i]);
  } else {
    const bool valid_slot = slot >= 0 && (long long)slot < (long long)block_size * num_blocks;
    if (valid_slot) {
      const long long base = ((long long)slot * kvheads + local_head) * kDim;
      const __nv_bfloat16* vsrc = qkv + packed + (long long)(qheads + kvheads + local_head) * kDim;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kcache[base + lane + 32 * i] = __float2bfloat16_rn(r[i]);
        vcache[base + lane + 32 * i] = vsrc[lane + 32 * i];
      }
    }
  }
}

// Rope table, same expression as the reference's rope_cache_kernel
// (kernels/kernels.cu:213-224) so the table is bit-identical.
__global__ void rope_cache_kernel(float* cache, int positions, int dim, float theta) {
  const int half = dim / 2;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (long long)positions * half;
       i += (long long)gridDim.x * blockDim.x) {
    const int position = int(i / half), pair = int(i % half);
    const float angle = position * powf(theta, -float(2 * pair) / dim);
    float s, c;
    sincosf(angle, &s, &c);
    cache[(long long)position * dim + pair] = c;
    cache[(long long)position * dim + half + pair] = s;
  }
}

}  // namespace rope_detail

cudaError_t launch_qkv_rope(cudaStream_t stream, bool cached, const void* qkv, const void* qw,
                            const void* kw, const int* positions, const int* slots, void* qout,
                            void* kc, void* vc, int rows, int qh, int kvh, int bs, int blocks,
                            float eps, float theta, const float* rope_cache, int max_positions) {
  using namespace rope_detail;
  const long long items = (long long)rows * (qh + kvh);
  const int warps_per_block = 8;
  const long long grid = (items + warps_per_block - 1) / warps_per_block;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  auto* q = static_cast<const __nv_bfloat16*>(qkv);
  auto* w0 = static_cast<const __nv_bfloat16*>(qw);
  auto* w1 = static_cast<const __nv_bfloat16*>(kw);
  auto* qo = static_cast<__nv_bfloat16*>(qout);
  auto* ko = static_cast<__nv_bfloat16*>(kc);
  auto* vo = static_cast<__nv_bfloat16*>(vc);
  if (cached)
    qkv_rope_kernel<true><<<unsigned(grid), 256, 0, stream>>>(q, w0, w1, positions, slots, qo, ko, vo, rows, qh,
                                                              kvh, bs, blocks, eps, 1.0f, rope_cache,
                                                              max_positions);
  else
    qkv_rope_kernel<false><<<unsigned(grid), 256, 0, stream>>>(q, w0, w1, positions, slots, qo, ko, vo, rows,
                                                               qh, kvh, bs, blocks, eps, theta, nullptr, 0);
  return cudaGetLastError();
}

cudaError_t launch_rope_cache(cudaStream_t stream, float* cache, int positions, int dim, float theta) {
  using namespace rope_detail;
  const long long elements = (long long)positions * (dim / 2);
  long long grid = (elements + 255) / 256;
  if (grid > 65535) grid = 65535;
  if (grid < 1) grid = 1;
  rope_cache_kernel<<<unsigned(grid), 256, 0, stream>>>(cache, positions, dim, theta);
  return cudaGetLastError();
}

}  // namespace nvb
