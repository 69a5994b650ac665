/*
 * nvb_attention.h — C ABI of the B200 (sm_100a) paged-attention library
 * `libnvb.so`. This is the drop-in boundary behind nano-vllm-rs's
 * `--attention-backend` seam.
 *
 * Every pointer except `stream` is a CUDA device pointer on the current
 * device. `stream` is a cudaStream_t owned by the caller. No attention entry
 * point allocates device memory, synchronizes the stream, or owns a context,
 * so their launches (nvb_paged_decode_static_scratch aside: see its own
 * comment) are safe inside CUDA-graph stream capture, with one exception:
 * the first launch that sees a new KV-cache base pointer encodes its TMA
 * descriptor on the host (no device work); do that first launch before
 * capture, as the reference engine does with its warm-up forward. The
 * multi-GPU set-up calls nvb_peer_buffer_* allocate and map memory (call
 * them once, outside capture), and nvb_paged_decode_gather takes a per-call
 * epoch, so a captured launch would replay a stale one: launch it directly.
 *
 * Layouts (identical to the reference):
 *   q, out           [total_q, q_heads, 128] bf16, contiguous
 *   k, v (per layer) [num_blocks, block_size, kv_heads, 128] bf16
 *   block_table      [batch, table_stride] int32, -1 marks an unused entry
 *   cu_q             [batch + 1] int32, cumulative query counts
 *   kv_lens          [batch] int32, NOT cumulative, includes this step
 *   slot_mapping     [rows] int32, slot = page * block_size + pos % block_size
 *
 * Return value: 0 on success, -1 on invalid host arguments, or a positive
 * cudaError_t for a launch error. The message is in a thread-local buffer
 * returned by nvb_last_error(). Asynchronous device faults surface at the
 * caller's next synchronization, as in the reference.
 */
#ifndef NVB_ATTENTION_H
#define NVB_ATTENTION_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Paged-KV attention, call-compatible with the reference's FlashAttention
 * adapter `nvr_flash_fwd` (kernels/flash_native/flash_native.h:22-27,
 * implementation kernels/flash_native/flash_native.cu:40-121; Rust binding
 * src/gpu.rs:181-202, caller src/gpu.rs:890-995).
 *
 *  - max_q == 1: decode. Exactly one query per sequence (total_q == batch).
 *    One CTA per (sequence, kv head, split) streams the sequence's KV pages
 *    through TMA; the whole GQA query group shares each KV tile. With
 *    num_splits > 1 the split partials go to lse_accum
 *    [num_splits, batch, q_heads] and out_accum [num_splits, batch, q_heads,
 *    128] (FP32) and a combine kernel writes `out`.
 *  - max_q > 1: varlen / chunked causal prefill. Queries of sequence b are
 *    the contiguous suffix of its KV context (bottom-right causal mask).
 *    Runs on tcgen05 tensor cores with TMEM accumulators. num_splits must
 *    be 1.
 *  - lse (natural-log softmax LSE) is written at [(b * q_heads + h) * max_q
 *    + i] for query i of sequence b.
 *
 * Limits: head_dim 128, block_size a positive multiple of 256, q_heads a
 * multiple of kv_heads, q_heads <= 256 (any GQA group, as the reference:
 * flash_native.cu:48-52), 1 <= num_splits <= 128. Unlike the reference (max_k <= 4096) the
 * context is bounded only by block_size * table_stride < 2^31.
 * Like the reference, page ids are trusted: a negative page id masks its
 * tokens, a page id past the end of the cache is undefined behaviour. Use
 * nvb_paged_fwd_ex to have out-of-range page ids masked as well.
 */
int nvb_paged_fwd(void* stream, const void* q, const void* k, const void* v, void* out,
                  const int* cu_q, const int* kv_lens, const int* block_table, int batch,
                  int total_q, int max_q, int max_k, int q_heads, int kv_heads, int block_size,
                  int table_stride, int num_splits, float* lse, float* lse_accum,
                  float* out_accum);

/* nvb_paged_fwd with the cache extent `num_blocks`: the TMA descriptors are
 * bounded by the cache and page ids outside [0, num_blocks) mask their
 * tokens (as the reference's native kernel does, kernels/kernels.cu:281-282).
 * This is the entry point the library's own host wrappers use. */
int nvb_paged_fwd_ex(void* stream, const void* q, const void* k, const void* v, void* out,
                     const int* cu_q, const int* kv_lens, const int* block_table, int batch,
                     int total_q, int max_q, int max_k, int q_heads, int kv_heads,
                     int block_size, int table_stride, int num_splits, float* lse,
                     float* lse_accum, float* out_accum, int num_blocks);

/* Split-KV decode that allocates nothing, for callers that cannot call
 * cudaMalloc (a plugin inside a host process that owns the CUDA allocator, a
 * fixed device-memory budget): the split partials live in a fixed array in
 * this library's device memory instead of caller-provided lse_accum /
 * out_accum. No counterpart in the reference. Decode only (one query per
 * sequence, total_q == batch); other arguments as nvb_paged_fwd_ex.
 * Limit: num_splits * batch * q_heads <= 16384 (about 8.1 MB held per GPU
 * until exit); larger calls return -1. All calls on a device share the array,
 * so calls that overlap on the GPU race; the first call in each CUDA context
 * (normally one per device) looks up the array's address and should come
 * before any stream capture. */
int nvb_paged_decode_static_scratch(void* stream, const void* q, const void* k, const void* v,
                                    void* out, const int* cu_q, const int* kv_lens,
                                    const int* block_table, int batch, int max_k, int q_heads,
                                    int kv_heads, int block_size, int table_stride,
                                    int num_splits, float* lse, int num_blocks);

/* Split count for decode, replacing `nvr_flash_num_splits`
 * (kernels/flash_native/flash_native.h:31-32, flash_native.cu:17-38).
 * A B200 heuristic: the most (sequence, kv head, split) CTAs that fit one
 * wave of 2 CTAs per SM, with at least 256 KV tokens per split.
 * Pass the physical SM count. Invalid arguments return 0. */
int nvb_num_splits(int batch, int q_heads, int kv_heads, int max_k, int num_sms);

/* Multi-GPU decode over kv-head shards (no counterpart in the reference,
 * which is single-GPU). One process per GPU of a node; rank r holds kv
 * heads [r*kv_heads, (r+1)*kv_heads) of the cache and passes its q
 * [batch, q_heads, 128] (the query heads of those kv heads). The split-KV
 * combine stores each result into every rank's output
 * [batch, world*q_heads, 128] at head offset r*q_heads (peer stores over
 * NVLink), then a one-warp barrier exchanges `epoch` with every rank; when
 * the call's work on `stream` is done, every rank's contributions are in this
 * rank's output. Arguments as nvb_paged_fwd_ex (max_q = 1, no lse) plus:
 *   out_local   [batch, q_heads, 128] BF16 scratch (used when num_splits == 1)
 *   peer_out    host array of `world` device pointers: each rank's output
 *   peer_flag   host array of `world` device pointers: each rank's flags,
 *               at least `world` uint32 starting at 0 (one slot per rank)
 *   epoch       strictly increasing per call (1, 2, ...), the same on every rank
 * Every rank must make the call with the same epoch; a rank that does not
 * leaves the others' barrier to give up after about two seconds, recording
 * device error 7 (nvb_device_error). Output buffers are written by all
 * ranks: alternate two of them between steps, and read step n's output (or
 * enqueue its readers on `stream`) before this rank's next call. A peer one
 * step ahead stores step n + 2 into the same buffer as soon as this rank's
 * step n + 1 has exchanged its epoch, which is before work enqueued after
 * that call runs. The same holds for the two output sets of the capturable
 * form below. */
int nvb_paged_decode_gather(void* stream, const void* q, const void* k, const void* v, void* out_local,
                            const int* cu_q, const int* kv_lens, const int* block_table, int batch, int max_k,
                            int q_heads, int kv_heads, int block_size, int table_stride, int num_blocks,
                            int num_splits, float* lse_accum, float* out_accum, void* const* peer_out,
                            unsigned int* const* peer_flag, int world, int rank, unsigned int epoch);

/* The same step in a form that a CUDA graph can capture once and replay
 * (no host argument changes between steps; no counterpart in the reference).
 * The epoch lives in device memory: peer_flag[rank] needs world + 2 uint32
 * (starting at 0): slot `world` is this rank's step counter, advanced at the
 * end of each step, and slot world + 1 a count of finished combine CTAs (the
 * last one runs the epoch exchange, so a step is two launches, decode and
 * combine, and no separate barrier). Step n (n = 1, 2, ...)
 * writes its results into output set n & 1: peer_out1[p] for odd n,
 * peer_out0[p] for even n, each rank's [batch, world*q_heads, 128] BF16.
 * Every rank must run the same number of steps in the same order; do not
 * mix calls of this form and of nvb_paged_decode_gather on one flag set. */
int nvb_paged_decode_gather_capturable(void* stream, const void* q, const void* k, const void* v, void* out_local,
                                       const int* cu_q, const int* kv_lens, const int* block_table, int batch,
                                       int max_k, int q_heads, int kv_heads, int block_size, int table_stride,
                                       int num_blocks, int num_splits, float* lse_accum, float* out_accum,
                                       void* const* peer_out0, void* const* peer_out1,
                                       unsigned int* const* peer_flag, int world, int rank);

/* Device buffers shared between the ranks of a node through CUDA IPC (the
 * outputs and flags of nvb_paged_decode_gather). create: cudaMalloc `bytes`
 * (zeroed) and write its 64-byte IPC handle; open: map a peer's handle;
 * close: unmap a peer's mapping; free: release this rank's buffer. */
int nvb_peer_buffer_create(size_t bytes, void** ptr, void* ipc_handle);
int nvb_peer_buffer_open(const void* ipc_handle, void** ptr);
int nvb_peer_buffer_close(void* ptr);
int nvb_peer_buffer_free(void* ptr);

/* Thread-local message for the last failing call on this thread
 * (kernels/flash_native/flash_native.cu:15, kernels/kernels.cu:28). */
const char* nvb_last_error(void);

/* Native-backend-compatible causal paged GQA, replacing `nv_attention`
 * (kernels/kernels.cu:475-485; Rust wrapper src/gpu.rs:829-887) with an
 * explicit stream instead of the reference's Context*. Row r attends to
 * positions[r] + 1 keys of block-table row seq_indices[r]; rows whose
 * sequence or context is invalid get zero output, as in the reference.
 * head_dim 128 (block_size a multiple of 32) runs on the tiled decode;
 * other head sizes from 1 to 512 (any block size) run on a generic CUDA-core
 * kernel, as the reference dispatches head sizes (kernels.cu:226-271,
 * 475-485). Other values are rejected with -1. Requires no scratch. */
int nvb_attention(void* stream, const void* q, const void* kcache, const void* vcache,
                  const int* positions, const int* seq_indices, const int* tables, void* out,
                  int rows, int q_heads, int kv_heads, int head_dim, int block_size,
                  int num_blocks, int table_stride, int batch, int max_context);

/* nvb_attention with split-KV, argument-compatible with the reference's
 * research entry `nv_attention_splitkv_candidate`
 * (kernels/decode_candidate.cuh:111-202, 247): (scratch, partitions)
 * appended. scratch holds rows * q_heads * partitions * (128 + 2) floats;
 * 1 <= partitions <= 128; partitions > 1 needs head_dim 128. */
int nvb_attention_splitkv(void* stream, const void* q, const void* kcache, const void* vcache,
                          const int* positions, const int* seq_indices, const int* tables,
                          void* out, int rows, int q_heads, int kv_heads, int head_dim,
                          int block_size, int num_blocks, int table_stride, int batch,
                          int max_context, float* scratch, int partitions);

/* Fused per-head Q/K RMSNorm + rotate-half RoPE + paged KV store, replacing
 * `nv_qkv_rope_cached` (kernels/kernels.cu:166-211, 474; Rust wrapper
 * src/gpu.rs:775-825) with an explicit stream. qkv is [rows, qh + 2*kvh,
 * dim] bf16 (q heads, then k heads, then v heads). Q goes to qout [rows, qh,
 * dim]; rotated K and copied V go to cache slot slots[row] (slots outside
 * [0, block_size * num_blocks) are skipped). rope_cache is [max_positions,
 * dim] FP32 with cos in columns [0, dim/2) and sin in [dim/2, dim);
 * positions outside [0, max_positions) use cos 1, sin 0. Bit-identical to
 * the reference kernel. dim must be 128. */
int nvb_qkv_rope_cached(void* stream, const void* qkv, const void* q_weight,
                        const void* k_weight, const int* positions, const int* slots,
                        void* qout, void* kcache, void* vcache, int rows, int q_heads,
                        int kv_heads, int head_dim, int block_size, int num_blocks, float eps,
                        const float* rope_cache, int max_positions);

/* Same, computing the rotation angle in-kernel from theta, replacing
 * `nv_qkv_rope` (kernels/kernels.cu:472). */
int nvb_qkv_rope(void* stream, const void* qkv, const void* q_weight, const void* k_weight,
                 const int* positions, const int* slots, void* qout, void* kcache, void* vcache,
                 int rows, int q_heads, int kv_heads, int head_dim, int block_size,
                 int num_blocks, float eps, float theta);

/* Builds the FP32 cos/sin table [positions, dim] for nvb_qkv_rope_cached,
 * replacing `nv_rope_cache` (kernels/kernels.cu:213-224, 473). */
int nvb_rope_cache(void* stream, float* cache, int positions, int head_dim, float theta);

/* CUDA-graph helpers on a caller stream, replacing nv_capture_begin /
 * nv_capture_end / nv_capture_abort / nv_graph_replay / nv_graph_destroy
 * (kernels/kernels.cu:80-97). Capture mode is thread-local, as in the
 * reference. *graph receives a cudaGraphExec_t. */
int nvb_capture_begin(void* stream);
int nvb_capture_end(void* stream, void** graph);
void nvb_capture_abort(void* stream);
int nvb_graph_replay(void* graph, void* stream);
void nvb_graph_destroy(void* graph);

/* Device-side error word written by bounded pipeline waits (0 = none).
 * Reading it synchronizes the device; it is a diagnostic, not for the
 * step loop. No counterpart in the reference, whose kernels do not spin. */
int nvb_device_error(int* code);
int nvb_clear_device_error(void);

/* Library version string. */
const char* nvb_version(void);

#ifdef __cplusplus
}
#endif

#endif /* NVB_ATTENTION_H */
