/*
 * nvb_host.h — C ABI of libnvb_host.so, the host-side pieces of the paged
 * attention path: the integer metadata the kernels consume. Plain C++, no
 * CUDA: every function here runs on the CPU.
 *
 * These restate the reference's Rust host code on the path (the Rust host
 * cannot be built in this image): batch layout and page allocation
 * (src/runtime.rs), the attention metadata derived from it and its packed
 * upload (src/model.rs). Integer results must be bit-exact with the
 * reference; error messages follow the reference's wording.
 *
 * Return value convention: 0 on success, -1 on invalid input with a
 * thread-local message in nvbh_last_error().
 */
#ifndef NVB_HOST_H
#define NVB_HOST_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

const char* nvbh_last_error(void);

/* One forward pass's flattened input, the reference's `Batch`
 * (src/runtime.rs:17-29). Arrays are borrowed. */
typedef struct NvbhBatch {
  const int32_t* token_ids;          /* [rows] */
  const int32_t* positions;          /* [rows] */
  const int32_t* sequence_ids;       /* [rows], index into block-table rows */
  const int32_t* slot_mapping;       /* [rows] */
  size_t rows;
  const int32_t* block_tables;       /* [sequences * table_stride], -1 padded */
  size_t block_tables_len;
  size_t table_stride;
  const int32_t* last_token_indices; /* [samples] */
  const float* temperatures;         /* [samples] */
  const uint64_t* seeds;             /* [samples] */
  size_t samples;
  int is_decode;
} NvbhBatch;

/* cu_q / kv_lens / max_q for the paged attention ABI from a batch's
 * positions and sequence ids, replacing `flash_metadata`
 * (src/model.rs:234-267). cu_q has sequences + 1 entries, kv_lens
 * sequences. Rejects non-consecutive positions, empty or out-of-order
 * groups and KV-length overflow, as the reference does. */
int nvbh_flash_metadata(const int32_t* positions, const int32_t* sequence_ids, size_t rows,
                        size_t sequences, int32_t* cu_q, int32_t* kv_lens, size_t* max_q);

/* Fixed 8-byte-aligned ranges of the single packed metadata upload,
 * replacing `MetadataLayout` (src/model.rs:271-321). start[i] / end[i] are
 * byte offsets for the NVBH_META_* fields. */
enum {
  NVBH_META_TOKENS = 0,
  NVBH_META_POSITIONS,
  NVBH_META_SEQUENCES,
  NVBH_META_SLOTS,
  NVBH_META_TABLES,
  NVBH_META_LAST_INDICES,
  NVBH_META_TEMPERATURES,
  NVBH_META_SEEDS,
  NVBH_META_CU_Q,
  NVBH_META_KV_LENS,
  NVBH_META_FIELDS
};
typedef struct NvbhMetadataLayout {
  size_t start[NVBH_META_FIELDS];
  size_t end[NVBH_META_FIELDS];
  size_t bytes;
} NvbhMetadataLayout;

int nvbh_metadata_layout(size_t tokens, size_t sequences, size_t table_stride,
                         NvbhMetadataLayout* out);

/* Packs a batch into the staging buffer, replacing `MetadataLayout::pack`
 * (src/model.rs:323-358): table rows are padded to the layout's stride with
 * 0xFF bytes (-1). cu_q / kv_lens, if non-null, are written to their ranges
 * as src/model.rs:935-945 does. */
int nvbh_metadata_pack(const NvbhMetadataLayout* layout, uint8_t* staging, size_t staging_bytes,
                       const NvbhBatch* batch, size_t sequences, size_t table_stride,
                       const int32_t* cu_q, const int32_t* kv_lens);

/* Model capacities for batch validation (src/model.rs:51-181 options). */
typedef struct NvbhLimits {
  size_t max_batch_tokens;
  size_t max_sequences;
  size_t max_model_len;
  size_t block_size;
  size_t num_blocks;
  size_t table_stride;
  size_t vocab_size;
} NvbhLimits;

/* Host invariants before any device work, replacing
 * `QwenModel::validate_batch` (src/model.rs:820-921): slot agrees with the
 * block table, slots unique, every causal page valid. Outputs rows,
 * sequences and samples. */
int nvbh_validate_batch(const NvbhBatch* batch, const NvbhLimits* limits, size_t* rows,
                        size_t* sequences, size_t* samples);

/* Reference-counted page pool with exact-token prefix keys and LRU reuse,
 * replacing `BlockPool` (src/runtime.rs:192-296). */
typedef struct NvbhBlockPool NvbhBlockPool;
NvbhBlockPool* nvbh_pool_create(size_t num_blocks);
void nvbh_pool_destroy(NvbhBlockPool* pool);
/* Free page with the lowest (has cached prefix, last used) key, its prefix
 * key dropped; -1 when every page is referenced. */
int nvbh_pool_allocate(NvbhBlockPool* pool);
void nvbh_pool_release(NvbhBlockPool* pool, int block);
int nvbh_pool_find(const NvbhBlockPool* pool, const uint32_t* tokens, size_t n);
int nvbh_pool_find_and_retain(NvbhBlockPool* pool, const uint32_t* tokens, size_t n);
void nvbh_pool_publish(NvbhBlockPool* pool, int block, const uint32_t* prefix, size_t n);
size_t nvbh_pool_available(const NvbhBlockPool* pool);
size_t nvbh_pool_in_use(const NvbhBlockPool* pool);
size_t nvbh_pool_references(const NvbhBlockPool* pool, int block);
size_t nvbh_pool_cached_keys(const NvbhBlockPool* pool);
void nvbh_pool_clear_cache(NvbhBlockPool* pool);
/* Test hook: files `block` under the hash of another prefix, simulating a
 * hash collision (src/runtime/tests.rs:213-234 does the same in Rust). */
void nvbh_pool_force_hash_entry(NvbhBlockPool* pool, const uint32_t* prefix, size_t n, int block);

/* One sequence's slice of a forward pass (the reference's Segment plus the
 * sequence fields make_batch reads, src/runtime.rs:355-358, 728-777). */
typedef struct NvbhSegment {
  const uint32_t* tokens;  /* the sequence's tokens so far (prompt + generated) */
  size_t num_tokens;
  const int32_t* blocks;   /* physical pages held by the sequence */
  size_t num_blocks;
  size_t start, end;       /* positions computed by this pass: [start, end) */
  int sample;              /* sample a token after position end - 1 */
  uint64_t request_id;
  size_t generated;        /* tokens generated so far */
  float temperature;
} NvbhSegment;

/* Output arrays of make_batch; *_cap are capacities, the counts are outputs. */
typedef struct NvbhBatchOut {
  int32_t* token_ids;
  int32_t* positions;
  int32_t* sequence_ids;
  int32_t* slot_mapping;
  size_t rows_cap;
  int32_t* block_tables;
  size_t tables_cap;
  int32_t* last_token_indices;
  float* temperatures;
  uint64_t* seeds;
  size_t samples_cap;
  size_t rows;
  size_t table_stride;
  size_t samples;
} NvbhBatchOut;

/* Flattens segments into a batch, replacing `LlmEngine::make_batch`
 * (src/runtime.rs:728-777): slot = page[pos / block_size] * block_size +
 * pos % block_size, tables padded with -1 to the largest page count. */
int nvbh_make_batch(const NvbhSegment* segments, size_t n, size_t block_size, uint64_t seed,
                    NvbhBatchOut* out);

/* Per-request, per-step sampling seed (src/runtime.rs:782-790). */
uint64_t nvbh_sampling_seed(uint64_t base, uint64_t request_id, uint64_t generated);

#ifdef __cplusplus
}
#endif

#endif /* NVB_HOST_H */
