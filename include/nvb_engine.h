/*
 * nvb_engine.h — C ABI of the continuous-batching engine and the Qwen3 model
 * runner around the paged-attention path.
 *
 * Two libraries:
 *   libnvb_host.so   nvbe_engine_*: the scheduler (plain C++, no CUDA). It
 *                    restates the reference's LlmEngine (src/runtime.rs:
 *                    358-777): admission against free KV pages, prefix
 *                    reuse, chunked prefill under a token budget, preemption
 *                    with recomputation, per-request sampling seeds. It
 *                    drives any model runner through NvbeRunFn, the
 *                    reference's ModelRunner trait (src/runtime.rs:41-49).
 *   libnvb_model.so  nvbe_model_*: the Qwen3 forward (src/model.rs:635-818)
 *                    on one GPU with this library's attention kernels
 *                    (libnvb.so) behind the attention seam, the reference's
 *                    device-side batch layout (src/model.rs:271-359), and
 *                    CUDA-graph replay of decode steps (src/model.rs:959-974).
 *
 * Return value convention: 0 on success, -1 on invalid input, or a positive
 * CUDA / cuBLAS status; the message is in a thread-local buffer
 * (nvbe_engine_last_error for the engine, nvbe_model_last_error for the
 * model).
 */
#ifndef NVB_ENGINE_H
#define NVB_ENGINE_H

#include <stddef.h>
#include <stdint.h>

#include "nvb_host.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ scheduler */

/* SchedulerConfig (src/runtime.rs:73-121). eos_token_id < 0: no EOS token. */
typedef struct NvbeSchedulerConfig {
  size_t block_size;
  size_t num_blocks;
  size_t max_sequences;
  size_t max_model_len;
  size_t max_batch_tokens;
  int prefix_caching;
  int64_t eos_token_id;
  /* 0: prefill and decode run in separate forwards, as the reference does
   * (src/runtime.rs:557-565). 1: one forward takes every running
   * sequence's decode token first, then prefill chunks under the same
   * max_batch_tokens budget, so admitting a request does not stall decoding
   * (the attention kernels take mixed query lengths in one launch). */
  int mixed_batches;
} NvbeSchedulerConfig;

/* Request (src/runtime.rs:51-71). The prompt is borrowed for the call. */
typedef struct NvbeRequest {
  uint64_t id;
  const uint32_t* prompt_token_ids;
  size_t prompt_len;
  size_t max_tokens;
  float temperature;
  int ignore_eos;
} NvbeRequest;

enum { NVBE_FINISH_LENGTH = 0, NVBE_FINISH_EOS = 1 };

/* RequestOutput (src/runtime.rs:130-143), written into caller-owned arrays:
 * token_ids and inter_token_latencies_ms need max_tokens entries each
 * (inter_token_latencies_ms may be null). */
typedef struct NvbeRequestOutput {
  uint32_t* token_ids;
  size_t num_tokens;
  size_t prompt_tokens;
  size_t cached_tokens;
  double ttft_ms;
  double latency_ms;
  double* inter_token_latencies_ms;
  size_t num_gaps;
  int finish_reason;
} NvbeRequestOutput;

/* RunStats (src/runtime.rs:145-170). */
typedef struct NvbeRunStats {
  double elapsed_seconds;
  size_t input_tokens;
  size_t output_tokens;
  double output_tokens_per_second;
  size_t total_requests;
  size_t cached_tokens;
  size_t cache_hits;
  size_t prefill_tokens;
  size_t decode_tokens;
  size_t prefill_steps;
  size_t decode_steps;
  double prefill_seconds;
  double decode_seconds;
  size_t preemptions;
  size_t peak_kv_blocks;
  double mean_ttft_ms;
  double mean_latency_ms;
  double mean_inter_token_latency_ms;
  /* Forwards that held both decode rows and prefill rows (mixed_batches);
   * their rows count in decode_tokens / prefill_tokens by kind and their
   * time in mixed_seconds only. */
  size_t mixed_steps;
  double mixed_seconds;
} NvbeRunStats;

/* One forward pass: fill sampled[batch->samples]. Nonzero = failure. */
typedef int (*NvbeRunFn)(void* runner, const NvbhBatch* batch, uint32_t* sampled);
/* Wait for the runner's device work (may be null). Nonzero = failure. */
typedef int (*NvbeSyncFn)(void* runner);

typedef struct NvbeEngine NvbeEngine;

/* SchedulerConfig::validate (src/runtime.rs:99-121). */
int nvbe_scheduler_config_validate(const NvbeSchedulerConfig* config);
int nvbe_engine_create(const NvbeSchedulerConfig* config, NvbeRunFn run, NvbeSyncFn sync, void* runner,
                       NvbeEngine** out);
void nvbe_engine_destroy(NvbeEngine* engine);
/* LlmEngine::generate (src/runtime.rs:386-409): runs every request to
 * completion; outputs[i] belongs to requests[i]. A runner failure releases
 * every page, drops the prefix cache and makes the engine refuse later
 * calls, as the reference does. */
int nvbe_engine_generate(NvbeEngine* engine, const NvbeRequest* requests, size_t n, uint64_t seed,
                         NvbeRequestOutput* outputs, NvbeRunStats* stats);
/* LlmEngine::clear_prefix_cache (src/runtime.rs:379-384). */
int nvbe_engine_clear_prefix_cache(NvbeEngine* engine);
size_t nvbe_engine_blocks_in_use(const NvbeEngine* engine);
size_t nvbe_engine_cached_keys(const NvbeEngine* engine);
const char* nvbe_engine_last_error(void);

/* ---------------------------------------------------------- model runner */

/* The Qwen3 fields of config.json the forward uses (src/model.rs:19-49). */
typedef struct NvbeModelConfig {
  int hidden_size;
  int intermediate_size;
  int num_hidden_layers;
  int num_attention_heads;
  int num_key_value_heads;
  int head_dim;
  int vocab_size;
  float rms_norm_eps;
  float rope_theta;
  int tie_word_embeddings;
} NvbeModelConfig;

/* ModelOptions (src/model.rs:151-181); the attention backend is this
 * library's (the paged kernels of libnvb.so). */
typedef struct NvbeModelOptions {
  int device;
  int block_size;
  int num_blocks;
  int max_batch_tokens;
  int max_sequences;
  int max_model_len;
  int cuda_graphs;
  /* 1: projections of small forwards (decode steps of up to 8 sequences,
   * and up to 64 for projections of at most 2048 outputs, where it was
   * measured faster) run on this library's tcgen05 GEMM (nvbe_layer_gemm,
   * SiLU fused into the gate/up projection), and steps sampling at most 4
   * rows run the LM head with the sampler fused (nvbe_layer_gemm_sample);
   * larger ones use cuBLAS. 0: cuBLAS throughout. */
  int tc_gemms;
} NvbeModelOptions;

/* Borrowed BF16 device weights, row-major [out, in] like the checkpoint
 * (src/model.rs:431-504): per layer qkv = q_proj ; k_proj ; v_proj rows and
 * gate_up = gate_proj ; up_proj rows. lm_head may be null when the
 * embeddings are tied. Each per-layer field is an array of
 * num_hidden_layers device pointers. */
typedef struct NvbeModelWeights {
  const void* embedding;        /* [vocab, hidden] */
  const void* final_norm;       /* [hidden] */
  const void* lm_head;          /* [vocab, hidden] or null */
  const void* const* input_norm;     /* [hidden] */
  const void* const* qkv;            /* [(qh + 2 kvh) * dim, hidden] */
  const void* const* q_norm;         /* [dim] */
  const void* const* k_norm;         /* [dim] */
  const void* const* o_proj;         /* [hidden, qh * dim] */
  const void* const* post_norm;      /* [hidden] */
  const void* const* gate_up;        /* [2 * intermediate, hidden] */
  const void* const* down;           /* [hidden, intermediate] */
} NvbeModelWeights;

typedef struct NvbeModel NvbeModel;

/* QwenModel::load minus the checkpoint reader (src/model.rs:381-591):
 * allocates the paged K/V caches (num_blocks * block_size tokens per layer)
 * and the workspace for max_batch_tokens rows, builds the RoPE table, and
 * creates its own stream and cuBLAS handle on `device`. */
int nvbe_model_create(const NvbeModelConfig* config, const NvbeModelOptions* options,
                      const NvbeModelWeights* weights, NvbeModel** out);
void nvbe_model_destroy(NvbeModel* model);
/* ModelRunner::run (src/model.rs:924-1003), an NvbeRunFn: validates the
 * batch, uploads its packed metadata once (asynchronously, from pinned
 * memory), runs the forward (decode batches replay a CUDA graph per batch
 * size when cuda_graphs is set) and returns the sampled token ids. */
int nvbe_model_run(void* model, const NvbhBatch* batch, uint32_t* sampled);
/* An NvbeSyncFn: waits for the model's stream. */
int nvbe_model_sync(void* model);
/* BF16 logits of the sampled rows of the latest run, [samples, vocab]
 * (QwenModel::last_logits, src/model.rs:608-626); a diagnostic copy. */
int nvbe_model_last_logits(NvbeModel* model, uint16_t* out, size_t capacity, size_t* samples);
/* Device pointers of layer `layer`'s K and V caches ([num_blocks,
 * block_size, kv_heads, head_dim] BF16), for tests. */
int nvbe_model_kv_cache(NvbeModel* model, int layer, void** k, void** v);
/* The model's CUDA stream (a cudaStream_t). */
void* nvbe_model_stream(NvbeModel* model);
size_t nvbe_model_graph_count(const NvbeModel* model);
const char* nvbe_model_last_error(void);

/* ------------------------------------------------ per-layer kernels
 * The forward's non-attention kernels, each replacing the reference's entry
 * point of the same layer (kernels/kernels.cu:470-500) with an explicit
 * cudaStream_t instead of its Context*. BF16 outputs are bit-identical to
 * the reference kernels'. Buffers are device pointers; rows-by-hidden
 * arrays are contiguous, 16-byte aligned where vector access needs it. */
/* nv_embedding: out[r] = weight[tokens[r]] (zero for ids outside [0, vocab)). */
int nvbe_layer_embedding(void* stream, const int* tokens, const void* weight, void* out, int rows, int hidden,
                         int vocab);
/* nv_rms: out = x * rsqrt(mean(x^2) + eps) * weight. */
int nvbe_layer_rms(void* stream, const void* x, const void* weight, void* out, int rows, int hidden, float eps);
/* nv_add_rms: residual += x (stored BF16), out = rms(residual) * weight. */
int nvbe_layer_add_rms(void* stream, const void* x, void* residual, const void* weight, void* out, int rows,
                       int hidden, float eps);
/* nv_silu: out[r] = silu(packed[r, :I]) * packed[r, I:2I]. */
int nvbe_layer_silu_mul(void* stream, const void* packed, void* out, int rows, int intermediate);
/* nv_gather: out[r] = x[indices[r]] (zero for indices outside [0, input_rows)). */
int nvbe_layer_gather(void* stream, const void* x, const int* indices, void* out, int rows, int hidden,
                      int input_rows);
/* Decode-shaped GEMM on tcgen05 tensor cores, replacing the reference's
 * cublasGemmEx for M <= 256 rows (kernels/kernels.cu:98-106):
 * y[M, N] = x[M, K] w[N, K]^T, BF16 in and out, FP32 accumulation, K split
 * over a thread-block cluster and summed in a fixed order (deterministic).
 * silu = 1: w holds gate rows then up rows ([2I, K], N = 2I) and
 * y[M, I] = silu(gate) * up with the reference's SiLU arithmetic on the
 * BF16-rounded gate and up (kernels/kernels.cu:355-364). K a multiple of
 * 64, N a multiple of 4 (8 with silu), pointers 16-byte aligned. The FP32
 * split-K partials go through `workspace` (at least
 * nvbe_gemm_workspace_bytes(M, N, K, silu) bytes; the call allocates
 * nothing). */
size_t nvbe_gemm_workspace_bytes(int M, int N, int K, int silu);
int nvbe_layer_gemm(void* stream, const void* x, const void* w, void* y, int M, int N, int K, int silu,
                    void* workspace, size_t workspace_bytes);
/* The decode GEMM's device error word: 0, or 1 when a pipeline wait gave up
 * (about two seconds); -1 if it cannot be read. */
int nvbe_gemm_device_error(void);

/* The LM head with Gumbel-max sampling fused into its epilogue (the
 * reference runs cublasGemmEx, kernels/kernels.cu:98-106, then its sampler,
 * kernels/kernels.cu:378-466): logits[M, N] = x[M, K] w[N, K]^T (BF16, as
 * nvbe_layer_gemm rounds them) and out[M] = the sampled tokens, picked with
 * the reference's SplitMix64 Gumbel stream exactly as nvbe_layer_sample
 * picks them from those logits. The partial buffers hold
 * M * nvbe_gemm_sample_tiles(N) entries each. M <= 256, K a multiple of
 * 64, N of 4. */
int nvbe_gemm_sample_tiles(int vocab);
int nvbe_layer_gemm_sample(void* stream, const void* x, const void* w, void* logits, int M, int N, int K,
                           const float* temperatures, const uint64_t* seeds, int* out, float* partial_scores,
                           int* partial_indices);

/* nv_sample_parallel: Gumbel-max sampling with the reference's SplitMix64
 * stream (temperature 0: argmax), ties to the lowest token id. The partial
 * buffers hold rows * nvbe_sample_partitions(vocab) entries each. */
int nvbe_sample_partitions(int vocab);
int nvbe_layer_sample(void* stream, const void* logits, const float* temperatures, const uint64_t* seeds, int* out,
                      float* partial_scores, int* partial_indices, int rows, int vocab);

#ifdef __cplusplus
}
#endif

#endif /* NVB_ENGINE_H */
