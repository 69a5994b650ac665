// Declarations shared by the kernel files of libnvb.so. The library is built
// as one translation unit (nvb_unity.cu) so that the device-global error
// word in common.cuh needs no relocatable device code.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "common.cuh"

namespace nvb {

// Query-row modes of the decode kernel.
enum DecodeMode : int {
  kModeDecode = 0,  // row b is sequence b's single query; lens = kv_lens
  kModeNative = 1,  // reference nv_attention form: lens = positions, seq_map = seq_indices
  kModeVarlen = 2,  // one CTA per query row of a varlen batch: seq_map = cu_q, lens = kv_lens
};

// Tokens per decode pipeline stage (TMA box {128, 1, kDecodeTile}).
constexpr int kDecodeTile = 32;

struct DecodeParams {
  const __nv_bfloat16* q;   // [rows, qh, 128]
  __nv_bfloat16* out;       // [rows, qh, 128]
  const int* lens;          // kv_lens[seq] (decode, varlen) or positions[row] (native)
  const int* seq_map;       // seq_indices[row] (native) or cu_q[batch + 1] (varlen)
  const int* block_table;   // [*, table_stride]
  float* lse;               // optional final LSE at (seq * qh + head) * max_q + i
  float* lse_accum;         // [splits, rows, qh]      (splits > 1)
  float* out_accum;         // [splits, rows, qh, 128] (splits > 1)
  int rows, qh, kvh, block_size, table_stride, num_blocks, batch, max_context;
  int num_splits, n_hgroups, max_q;
  int mode;
  int max_k;         // decode: the caller's bound on kv_lens (picks the decode schedule)
  float scale_log2;  // log2(e) / sqrt(128)
};

cudaError_t launch_decode(DecodeParams p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                          cudaStream_t stream);
// tcgen05 decode (decode_mma.cu); cudaErrorNotSupported when it does not
// cover the shape. Takes K/V tensor maps with a {64, 1, 128} 128B-swizzled
// box and the same maps with a {64, 1, 64} box for short last tiles.
cudaError_t launch_decode_mma(const DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                              const CUtensorMap& kmap_half, const CUtensorMap& vmap_half, cudaStream_t stream);
// Persistent form of the tcgen05 decode (decode_persistent.cu), for short
// contexts: same arguments plus the query map.
cudaError_t launch_decode_persistent(const DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                                     const CUtensorMap& kmap_half, const CUtensorMap& vmap_half,
                                     const CUtensorMap& qmap, cudaStream_t stream);
// Decode batches whose max_k is at most this use the persistent form.
constexpr int kPersistentMaxK = 2048;
int decode_group_chunk(int group);
// Split-KV combine of lse_accum / out_accum into out (and lse).
cudaError_t launch_combine(const DecodeParams& p, cudaStream_t stream);

cudaError_t launch_qkv_rope(cudaStream_t stream, bool cached, const void* qkv, const void* qw,
                            const void* kw, const int* positions, const int* slots, void* qout,
                            void* kc, void* vc, int rows, int qh, int kvh, int bs, int blocks,
                            float eps, float theta, const float* rope_cache, int max_positions);
cudaError_t launch_rope_cache(cudaStream_t stream, float* cache, int positions, int dim, float theta);

struct PrefillArgs {
  const void* q;
  const void* k;
  const void* v;
  void* out;
  const int* cu_q;
  const int* kv_lens;
  const int* block_table;
  float* lse;
  int batch, total_q, max_q, max_k, qh, kvh, block_size, table_stride, num_blocks;
};

// Host-side TMA descriptor helper (api.cu): 3-D BF16 map over
// [dims[2]][dims[1]][dims[0]], cached per thread, copied into *out.
int make_map_3d(const void* base, const uint64_t dims[3], const uint64_t strides[2],
                const uint32_t box[3], CUtensorMapSwizzle swizzle, CUtensorMap* out);

// Returns cudaErrorNotSupported when the tcgen05 path does not cover the shape.
// launch_prefill picks the kernel: pairs of query tiles per work item
// (prefill.cu) when a sequence can span more than one 128-row query tile,
// else one tile per item (prefill_tile.cu).
cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream);
cudaError_t launch_prefill_tile(const PrefillArgs& a, cudaStream_t stream);

// Per-context host caches. Device symbol addresses and kernel attributes
// belong to a CUDA context, not to a device: a host process may run this
// library under a context it created itself, or recreate the primary context
// (cudaDeviceReset). context_slot() maps the context current on the calling
// thread (identified by cuCtxGetId, which no later context reuses) to one of
// kContextSlots slots; `gen` is new each time a slot is handed to another
// context, so a value cached under a different gen is stale. Implemented in
// api.cu.
constexpr int kContextSlots = 64;
int context_slot(int* slot, unsigned* gen);

// Runs init() once per context: `seen` holds the gen init last ran under for
// each slot (zero-initialised; gens start at 1).
template <class F>
cudaError_t once_per_context(unsigned* seen, F&& init) {
  int slot = 0;
  unsigned gen = 0;
  if (int rc = context_slot(&slot, &gen)) return cudaError_t(rc);
  if (__atomic_load_n(&seen[slot], __ATOMIC_ACQUIRE) == gen) return cudaSuccess;
  const cudaError_t e = init();
  if (e == cudaSuccess) __atomic_store_n(&seen[slot], gen, __ATOMIC_RELEASE);
  return e;
}

// Native-form attention for head dimensions other than 128 (generic.cu).
cudaError_t launch_generic_attention(const void* q, const void* k, const void* v, void* out, const int* positions,
                                     const int* seq_indices, const int* tables, int rows, int qh, int kvh, int dim,
                                     int block_size, int num_blocks, int table_stride, int batch, int max_context,
                                     cudaStream_t stream);

}  // namespace nvb
