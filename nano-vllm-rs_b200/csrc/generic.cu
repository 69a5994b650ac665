// Native-form paged attention for head dimensions other than 128.
//
// Replaces the reference's head_dim dispatch of the native kernel
// (kernels/kernels.cu:475-485: templates for 32/64/128/256 and the generic
// `attention_kernel` of kernels.cu:226-271 otherwise). head_dim 128 runs on
// decode_kernel (decode.cu); every other size up to 512 runs here. It is a
// correctness path for models with other head sizes, not a tuned kernel: one
// warp per (row, query head), each lane owning head dimensions lane,
// lane + 32, ... (coalesced 64-byte K/V row reads), an online softmax over
// the row's tokens in order, FP32 accumulation, BF16 output.
//
// Semantics as the native path: row r attends to tokens [0, positions[r]]
// of sequence seq_indices[r]; a page id outside [0, num_blocks) masks its
// tokens; a row whose sequence index or context is invalid gets zeros.
#include "internal.cuh"

namespace nvb {

namespace generic_detail {

struct GenericParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* out;
  const int* positions;
  const int* seq_indices;
  const int* tables;
  int rows, qh, kvh, dim, block_size, num_blocks, table_stride, batch, max_context;
  float scale;
};

template <int kPer>  // head dimensions per lane: dim <= 32 * kPer
__global__ void __launch_bounds__(256) generic_attention_kernel(const GenericParams p) {
  const long long item = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);  // (row, head)
  const int lane = threadIdx.x & 31;
  if (item >= (long long)p.rows * p.qh) return;
  const int row = int(item / p.qh), head = int(item % p.qh);
  const int kvhead = head / (p.qh / p.kvh);
  __nv_bfloat16* dst = p.out + item * p.dim;
  const int seq = p.seq_indices[row];
  const long long ctx = (long long)p.positions[row] + 1;
  if (seq < 0 || seq >= p.batch || ctx < 1 || ctx > p.max_context ||
      ctx > (long long)p.table_stride * p.block_size) {
    for (int d = lane; d < p.dim; d += 32) dst[d] = __float2bfloat16(0.0f);
    return;
  }
  float qv[kPer], acc[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int d = lane + 32 * i;
    qv[i] = d < p.dim ? __bfloat162float(p.q[item * p.dim + d]) * p.scale : 0.0f;
    acc[i] = 0.0f;
  }
  const int* table = p.tables + (long long)seq * p.table_stride;
  float m = -INFINITY, l = 0.0f;
  for (int t = 0; t < int(ctx); ++t) {
    const int page = table[t / p.block_size];
    if (page < 0 || page >= p.num_blocks) continue;
    const long long base = (((long long)page * p.block_size + t % p.block_size) * p.kvh + kvhead) * p.dim;
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int d = lane + 32 * i;
      if (d < p.dim) s = fmaf(qv[i], __bfloat162float(p.k[base + d]), s);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    const float m_new = fmaxf(m, s);
    const float alpha = __expf(m - m_new);  // 0 on the first token (m = -inf)
    const float pr = __expf(s - m_new);
    l = l * alpha + pr;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int d = lane + 32 * i;
      const float vv = d < p.dim ? __bfloat162float(p.v[base + d]) : 0.0f;
      acc[i] = fmaf(pr, vv, acc[i] * alpha);
    }
    m = m_new;
  }
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int d = lane + 32 * i;
    if (d < p.dim) dst[d] = __float2bfloat16(acc[i] * inv);
  }
}

}  // namespace generic_detail

cudaError_t launch_generic_attention(const void* q, const void* k, const void* v, void* out, const int* positions,
                                     const int* seq_indices, const int* tables, int rows, int qh, int kvh, int dim,
                                     int block_size, int num_blocks, int table_stride, int batch, int max_context,
                                     cudaStream_t stream) {
  using namespace generic_detail;
  GenericParams p{static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                  static_cast<const __nv_bfloat16*>(v), static_cast<__nv_bfloat16*>(out), positions, seq_indices,
                  tables, rows, qh, kvh, dim, block_size, num_blocks, table_stride, batch, max_context,
                  1.0f / sqrtf(float(dim))};
  const long long items = (long long)rows * qh;
  const unsigned grid = unsigned((items + 7) / 8);
  if (dim <= 32)
    generic_attention_kernel<1><<<grid, 256, 0, stream>>>(p);
  else if (dim <= 64)
    generic_attention_kernel<2><<<grid, 256, 0, stream>>>(p);
  else if (dim <= 128)
    generic_attention_kernel<4><<<grid, 256, 0, stream>>>(p);
  else if (dim <= 256)
    generic_attention_kernel<8><<<grid, 256, 0, stream>>>(p);
  else
    generic_attention_kernel<16><<<grid, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace nvb
