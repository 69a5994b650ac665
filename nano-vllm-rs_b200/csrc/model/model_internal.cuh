// Kernel launchers shared by the files of libnvb_model.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace nvbm {

cudaError_t launch_embedding(cudaStream_t s, const int* tokens, const void* weight, void* out, int rows, int hidden,
                             int vocab, int sms);
// residual == nullptr: out = rms(x) * w; else residual += x (BF16) and out = rms(residual) * w.
cudaError_t launch_rms(cudaStream_t s, const void* x, void* residual, const void* weight, void* out, int rows,
                       int hidden, float eps);
cudaError_t launch_silu_mul(cudaStream_t s, const void* packed, void* out, int rows, int inter, int sms);
cudaError_t launch_gather(cudaStream_t s, const void* x, const int* indices, void* out, int rows, int hidden,
                          int input_rows, int sms);
int sample_partitions(int vocab);
cudaError_t launch_sample(cudaStream_t s, const void* logits, const float* temps, const uint64_t* seeds, int* out,
                          float* part_score, int* part_index, int rows, int vocab);

// Decode-shaped tcgen05 GEMM (gemm.cu): Y[M, N] = X[M, K] W[N, K]^T for
// M <= 256, or with silu, Y[M, N / 2] = silu(gate) * up where gate / up are
// the first / second halves of W's rows. Maps: gemm_weight_map (W [N, K],
// with the same `silu`) and gemm_input_map (X [M, K]). K a multiple of 64,
// N a multiple of 4 (8 with silu), ldy a multiple of 4.
int gemm_decode_max_rows();
// Whether the decode GEMM beats cuBLAS at this shape (the model's dispatch).
bool gemm_decode_preferred(int M, int N, int K);
// Whether the fused LM head + sampler beats cuBLAS + the sampler.
bool gemm_sample_preferred(int M);
int gemm_weight_map(const void* w, int N, int K, bool silu, CUtensorMap* out);
int gemm_input_map(const void* x, int M, int K, CUtensorMap* out);
// Split-K partials go through `ws` (gemm_decode_workspace bytes, 16-byte
// aligned), which callers keep for the launch's duration.
int gemm_decode_cluster(int M, int N, int K, bool silu, int sms);
size_t gemm_decode_workspace(int M, int N, int K, bool silu, int sms);
cudaError_t launch_gemm_decode(cudaStream_t stream, const CUtensorMap& wmap, const CUtensorMap& xmap, void* y,
                               int M, int N, int K, int ldy, bool silu, int sms, void* ws, size_t ws_bytes);
// The LM head with Gumbel-max sampling fused into its epilogue (gemm.cu):
// logits[M, N] (BF16, as the plain decode GEMM rounds them) and, per row, the
// best (score, token) of each 128-token tile in part_score / part_index
// [M][gemm_decode_tiles(N)], folded by launch_sample_combine (sample.cu).
int gemm_decode_tiles(int N);
cudaError_t launch_gemm_decode_sample(cudaStream_t stream, const CUtensorMap& wmap, const CUtensorMap& xmap,
                                      void* logits, int M, int N, int K, const float* temps, const uint64_t* seeds,
                                      float* part_score, int* part_index);
cudaError_t launch_sample_combine(cudaStream_t s, const float* part_score, const int* part_index, int* out, int rows,
                                  int parts);
// The decode GEMM's device error word (1: a pipeline wait gave up), or -1.
int gemm_decode_error();

}  // namespace nvbm
