// Kernel launchers shared by the files of libnvb_model.so.
#pragma once

#include <cuda_runtime.h>

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

}  // namespace nvbm
