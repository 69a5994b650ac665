// Varlen / chunked causal prefill over paged KV on tcgen05 tensor cores.
#include "internal.cuh"

namespace nvb {

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream) {
  (void)a;
  (void)stream;
  return cudaErrorNotSupported;
}

}  // namespace nvb
