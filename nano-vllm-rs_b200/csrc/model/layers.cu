// Non-attention layers of the Qwen3 forward (libnvb_model.so).
//
// These kernels sit around the attention seam; each is written so that its
// BF16 output is bit-identical to the reference's kernel of the same layer
// (kernels/kernels.cu), so that the engine's tokens differ from the
// reference engine's only through the attention kernels:
//   embedding        kernels.cu:125-130  plain row copy (0 for ids out of range)
//   rms / add_rms    kernels.cu:131-151  FP32 sum of squares in the same
//                    association (below), rsqrtf(mean + eps), BF16 stores of
//                    the updated residual and of (x * inv_rms) * w
//   silu_mul         kernels.cu:355-364  one BF16 rounding of
//                    gate / (1 + expf(-gate)) * up
//   gather           kernels.cu:365-370  row gather (0 for indices out of range)
// The layouts are this library's own: 128 threads per row for the norms
// (one warp per row for hidden sizes that are not a multiple of 256), 16-byte
// vector accesses elsewhere.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "model_internal.cuh"

namespace nvbm {

namespace {

__device__ __forceinline__ float bf(const __nv_bfloat16 x) { return __bfloat162float(x); }

// Embedding lookup: 8 BF16 (16 bytes) per thread.
__global__ void embedding_kernel(const int* __restrict__ tokens, const uint4* __restrict__ weight,
                                 uint4* __restrict__ out, int rows, int vec_per_row, int vocab) {
  const long long total = (long long)rows * vec_per_row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / vec_per_row, col = i - row * vec_per_row;
    const int token = tokens[row];
    out[i] = (token >= 0 && token < vocab) ? weight[(long long)token * vec_per_row + col] : make_uint4(0, 0, 0, 0);
  }
}

// RMSNorm over one row per warp.
//
// The sum of squares must round exactly as the reference's 256-thread block
// reduction does. There, thread t (0..255) accumulates x[t], x[t+256], ...
// in order with fused multiply-adds; each warp w then folds its 32 partials
// with a halving tree (lane i += lane i+16, +8, +4, +2, +1), and the eight
// warp sums are folded by the same tree with zeros in lanes 8..31, which
// leaves ((W0+W4)+(W2+W6)) + ((W1+W5)+(W3+W7)). Here lane l plays the
// reference threads l, l+32, ..., l+224 (partial p[m] for thread l + 32m),
// folds each p[m] across the warp with a butterfly (xor) tree, which adds
// the same pairs as the halving tree and leaves the result in every lane,
// and then combines the eight warp sums in the order above.
template <bool ADD>
__global__ void rms_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                           const __nv_bfloat16* __restrict__ weight, __nv_bfloat16* __restrict__ out, int rows,
                           int hidden, float eps) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const long long base = (long long)row * hidden;
  float p[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float s = 0.0f;
    for (int j = lane + 32 * m; j < hidden; j += 256) {
      float v = bf(x[base + j]);
      if (ADD) v += bf(residual[base + j]);
      s = __fmaf_rn(v, v, s);
    }
    p[m] = s;
  }
#pragma unroll
  for (int m = 0; m < 8; ++m)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) p[m] = __fadd_rn(p[m], __shfl_xor_sync(0xffffffffu, p[m], off));
  const float total = __fadd_rn(__fadd_rn(__fadd_rn(p[0], p[4]), __fadd_rn(p[2], p[6])),
                                __fadd_rn(__fadd_rn(p[1], p[5]), __fadd_rn(p[3], p[7])));
  const float inv_rms = rsqrtf(__fadd_rn(__fdiv_rn(total, float(hidden)), eps));
  for (int j = lane; j < hidden; j += 32) {
    float v = bf(x[base + j]);
    if (ADD) {
      v += bf(residual[base + j]);
      residual[base + j] = __float2bfloat16_rn(v);
    }
    const float normalized = __fmul_rn(v, inv_rms);
    out[base + j] = __float2bfloat16_rn(__fmul_rn(normalized, bf(weight[j])));
  }
}

// RMSNorm with 128 threads per row, for hidden = 256 * NV (NV <= 8): the
// same sum as rms_kernel, laid out for parallelism. Thread r plays the
// reference threads r and r + 128: it loads all 2 * NV of their elements at
// once (kept in registers for the output pass), forms each thread's partial
// with the same fused multiply-add chain, folds the two partials across its
// warp (reference warps w and w + 4 for warp w), and the eight warp sums
// meet in shared memory in the reference's order.
template <bool ADD, int NV>
__global__ void __launch_bounds__(128) rms_row_kernel(const __nv_bfloat16* __restrict__ x,
                                                      __nv_bfloat16* __restrict__ residual,
                                                      const __nv_bfloat16* __restrict__ weight,
                                                      __nv_bfloat16* __restrict__ out, int hidden, float eps) {
  // A decode GEMM launched after this kernel as a programmatic dependent may
  // start streaming its weights now; it waits for this grid before reading
  // the normed rows.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const long long base = (long long)blockIdx.x * hidden;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float v[2][NV];
#pragma unroll
  for (int s = 0; s < 2; ++s)
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = tid + 128 * s + 256 * i;
      float a = bf(x[base + j]);
      if (ADD) a += bf(residual[base + j]);
      v[s][i] = a;
    }
  float p[2];
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) acc = __fmaf_rn(v[s][i], v[s][i], acc);
    p[s] = acc;
  }
#pragma unroll
  for (int s = 0; s < 2; ++s)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) p[s] = __fadd_rn(p[s], __shfl_xor_sync(0xffffffffu, p[s], off));
  __shared__ float wsum[8];
  if (lane == 0) {
    wsum[warp] = p[0];
    wsum[warp + 4] = p[1];
  }
  __syncthreads();
  const float total = __fadd_rn(__fadd_rn(__fadd_rn(wsum[0], wsum[4]), __fadd_rn(wsum[2], wsum[6])),
                                __fadd_rn(__fadd_rn(wsum[1], wsum[5]), __fadd_rn(wsum[3], wsum[7])));
  const float inv_rms = rsqrtf(__fadd_rn(__fdiv_rn(total, float(hidden)), eps));
#pragma unroll
  for (int s = 0; s < 2; ++s)
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = tid + 128 * s + 256 * i;
      if (ADD) residual[base + j] = __float2bfloat16_rn(v[s][i]);
      const float normalized = __fmul_rn(v[s][i], inv_rms);
      out[base + j] = __float2bfloat16_rn(__fmul_rn(normalized, bf(weight[j])));
    }
}

template <bool ADD>
cudaError_t launch_rms_rows(cudaStream_t s, const __nv_bfloat16* x, __nv_bfloat16* residual,
                            const __nv_bfloat16* w, __nv_bfloat16* out, int rows, int hidden, float eps) {
  switch (hidden / 256) {
#define NVB_RMS_CASE(NV) \
  case NV:               \
    rms_row_kernel<ADD, NV><<<rows, 128, 0, s>>>(x, residual, w, out, hidden, eps); \
    break;
    NVB_RMS_CASE(1) NVB_RMS_CASE(2) NVB_RMS_CASE(3) NVB_RMS_CASE(4)
    NVB_RMS_CASE(5) NVB_RMS_CASE(6) NVB_RMS_CASE(7) NVB_RMS_CASE(8)
#undef NVB_RMS_CASE
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// SiLU(gate) * up over the packed [rows, 2 * inter] GEMM output, 8 outputs a thread.
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ packed, __nv_bfloat16* __restrict__ out, int rows,
                                int inter) {
  const int vec = inter / 8;
  const long long total = (long long)rows * vec;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / vec, c = (i - row * vec) * 8;
    const uint4 g4 = *reinterpret_cast<const uint4*>(packed + row * 2 * inter + c);
    const uint4 u4 = *reinterpret_cast<const uint4*>(packed + row * 2 * inter + inter + c);
    const __nv_bfloat16* g = reinterpret_cast<const __nv_bfloat16*>(&g4);
    const __nv_bfloat16* u = reinterpret_cast<const __nv_bfloat16*>(&u4);
    uint4 o4;
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(&o4);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float gate = bf(g[e]);
      const float activation = __fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate)));
      o[e] = __float2bfloat16_rn(__fmul_rn(activation, bf(u[e])));
    }
    *reinterpret_cast<uint4*>(out + row * inter + c) = o4;
  }
}

// out[i] = x[indices[i]] (16-byte vectors); rows with an invalid index are zero.
__global__ void gather_kernel(const uint4* __restrict__ x, const int* __restrict__ indices, uint4* __restrict__ out,
                              int rows, int vec_per_row, int input_rows) {
  const long long total = (long long)rows * vec_per_row;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / vec_per_row, col = i - row * vec_per_row;
    const int index = indices[row];
    out[i] = (index >= 0 && index < input_rows) ? x[(long long)index * vec_per_row + col] : make_uint4(0, 0, 0, 0);
  }
}

int grid_for(long long work, int threads, int sms) {
  const long long blocks = (work + threads - 1) / threads;
  const long long cap = (long long)sms * 16;
  return int(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

}  // namespace

cudaError_t launch_embedding(cudaStream_t s, const int* tokens, const void* weight, void* out, int rows, int hidden,
                             int vocab, int sms) {
  if (hidden % 8) return cudaErrorInvalidValue;
  const int vec = hidden / 8;
  embedding_kernel<<<grid_for((long long)rows * vec, 256, sms), 256, 0, s>>>(
      tokens, static_cast<const uint4*>(weight), static_cast<uint4*>(out), rows, vec, vocab);
  return cudaGetLastError();
}

cudaError_t launch_rms(cudaStream_t s, const void* x, void* residual, const void* weight, void* out, int rows,
                       int hidden, float eps) {
  constexpr int kWarps = 4;
  const int blocks = (rows + kWarps - 1) / kWarps;
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  const auto* wp = static_cast<const __nv_bfloat16*>(weight);
  auto* op = static_cast<__nv_bfloat16*>(out);
  if (hidden % 256 == 0 && hidden <= 2048 && rows <= 0x7fffffff) {
    return residual ? launch_rms_rows<true>(s, xp, static_cast<__nv_bfloat16*>(residual), wp, op, rows, hidden, eps)
                    : launch_rms_rows<false>(s, xp, nullptr, wp, op, rows, hidden, eps);
  }
  if (residual)
    rms_kernel<true><<<blocks, 32 * kWarps, 0, s>>>(xp, static_cast<__nv_bfloat16*>(residual), wp, op, rows, hidden,
                                                   eps);
  else
    rms_kernel<false><<<blocks, 32 * kWarps, 0, s>>>(xp, nullptr, wp, op, rows, hidden, eps);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(cudaStream_t s, const void* packed, void* out, int rows, int inter, int sms) {
  if (inter % 8) return cudaErrorInvalidValue;
  silu_mul_kernel<<<grid_for((long long)rows * (inter / 8), 256, sms), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(packed), static_cast<__nv_bfloat16*>(out), rows, inter);
  return cudaGetLastError();
}

cudaError_t launch_gather(cudaStream_t s, const void* x, const int* indices, void* out, int rows, int hidden,
                          int input_rows, int sms) {
  if (hidden % 8) return cudaErrorInvalidValue;
  const int vec = hidden / 8;
  gather_kernel<<<grid_for((long long)rows * vec, 256, sms), 256, 0, s>>>(
      static_cast<const uint4*>(x), indices, static_cast<uint4*>(out), rows, vec, input_rows);
  return cudaGetLastError();
}

}  // namespace nvbm
