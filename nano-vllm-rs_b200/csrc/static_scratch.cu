// Split-KV decode for callers that cannot allocate device memory.
//
// nvb_paged_fwd needs caller-owned FP32 scratch (lse_accum, out_accum) when it
// splits a sequence's keys across CTAs. Some callers have no way to provide
// it: a plugin loaded into a host process that owns the CUDA allocator (and
// forbids cudaMalloc outside it), code running under a memory budget fixed at
// start-up, or a caller between allocator lifetimes. This entry point keeps the
// split partials in a fixed array in the library's own device memory instead,
// so the caller passes only its inputs and outputs and nothing is allocated.
//
// Limits and sharing:
//  * The array holds at most kStaticPartials (split, sequence, query head)
//    partials: 16384 x 128 FP32 values plus 16384 LSEs, about 8.1 MB, held on
//    every GPU that loads the library until the process exits. Calls whose
//    num_splits * batch * q_heads exceeds that are rejected with -1.
//  * Every call on a device uses the same array and leaves its partials
//    there. Each call overwrites every partial it later reads (the decode
//    kernel writes all of them, empty splits included), so nothing has to be
//    cleared between calls. Two calls whose kernels overlap on the GPU (on
//    different streams, or from different host threads) race on the array;
//    serialise them on one stream.
//  * The first call in each CUDA context (normally one per device: the
//    primary context) looks up the array's device address with
//    cudaGetSymbolAddress (the host-side symbol is only a stand-in and must
//    never be passed to a kernel). Make that first call before any stream
//    capture.
#include <mutex>

#include "internal.cuh"

namespace nvb {

namespace static_scratch_detail {

constexpr int kStaticPartials = 16384;

static __device__ __align__(256) float g_static_partials[kStaticPartials * (128 + 1)];

std::mutex g_addr_mutex;
float* g_addr[kContextSlots] = {};
unsigned g_addr_gen[kContextSlots] = {};

// Device address of g_static_partials in the context current on this thread,
// looked up once per context: each context that loads the library has its
// own copy of the array, so an address from another context (another
// device, a context the host created itself, or a primary context that
// cudaDeviceReset replaced) must never be reused.
int static_scratch_address(float** out) {
  int slot = 0;
  unsigned gen = 0;
  if (int rc = context_slot(&slot, &gen)) return rc;
  std::lock_guard<std::mutex> lock(g_addr_mutex);
  if (g_addr_gen[slot] != gen) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_partials);
    if (e != cudaSuccess) return int(e);
    g_addr[slot] = static_cast<float*>(ptr);
    g_addr_gen[slot] = gen;
  }
  *out = g_addr[slot];
  return 0;
}

}  // namespace static_scratch_detail

}  // namespace nvb

extern "C" int nvb_paged_decode_static_scratch(void* stream, const void* q, const void* k, const void* v, void* out,
                                               const int* cu_q, const int* kv_lens, const int* block_table,
                                               int batch, int max_k, int q_heads, int kv_heads, int block_size,
                                               int table_stride, int num_splits, float* lse, int num_blocks) {
  using namespace nvb;
  using namespace nvb::api_detail;
  using namespace nvb::static_scratch_detail;
  g_last_error[0] = 0;
  if (num_splits < 1 || num_splits > 128 || batch <= 0 || q_heads <= 0)
    return fail("invalid static-scratch decode arguments");
  const long long partials = (long long)num_splits * batch * q_heads;
  if (num_splits > 1 && partials > kStaticPartials)
    return fail("static-scratch decode holds at most %d split partials; num_splits * batch * q_heads = %lld",
                kStaticPartials, partials);
  float* lse_accum = nullptr;
  float* out_accum = nullptr;
  if (num_splits > 1) {
    float* base = nullptr;
    const int rc = static_scratch_address(&base);
    if (rc) return cuda_status(cudaError_t(rc), "cudaGetSymbolAddress(static split-KV scratch)");
    out_accum = base;                                         // [splits][batch][q_heads][128]
    lse_accum = base + (size_t)kStaticPartials * 128;         // [splits][batch][q_heads]
  }
  return paged_fwd_impl(stream, q, k, v, out, cu_q, kv_lens, block_table, batch, batch, 1, max_k, q_heads,
                        kv_heads, block_size, table_stride, num_splits, lse, lse_accum, out_accum, num_blocks, true);
}
