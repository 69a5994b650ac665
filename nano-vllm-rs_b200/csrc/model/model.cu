// Qwen3 model runner on one GPU (include/nvb_engine.h, nvbe_model_*).
//
// The forward of the reference's QwenModel (src/model.rs:635-818) with this
// library's kernels at the attention seam: per layer
//   [add+]RMSNorm -> QKV GEMM -> nvb_qkv_rope_cached (Q/K norm, RoPE, paged
//   K/V store) -> nvb_paged_fwd_ex (tcgen05 prefill or split-KV decode) ->
//   O GEMM -> add+RMSNorm -> gate/up GEMM -> SiLU*up -> down GEMM,
// then the final norm, the last-row gather, the LM head and the sampler.
// GEMMs are cuBLAS (cublasGemmEx, BF16 in/out, FP32 accumulate), called
// exactly as the reference calls it (kernels/kernels.cu:98-106).
//
// One step (ModelRunner::run, src/model.rs:924-1003): validate the batch on
// the host, derive cu_q / kv_lens, pack everything into one pinned staging
// buffer with the reference's layout (src/model.rs:271-359) and upload it
// with one asynchronous copy; decode batches replay a CUDA graph captured
// once per batch size after a warm-up forward (src/model.rs:959-974); the
// sampled ids come back with one asynchronous copy and one stream sync. The
// reference synchronises after the upload as well (kernels/kernels.cu:68-72);
// here the copy is ordered on the stream, and the staging buffer is not
// rewritten before the step's sync.
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <new>
#include <unordered_map>
#include <vector>

#include "model_internal.cuh"
#include "nvb_attention.h"
#include "nvb_engine.h"

namespace {

thread_local char g_model_error[512] = {};

int mfail(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  std::vsnprintf(g_model_error, sizeof(g_model_error), fmt, args);
  va_end(args);
  return -1;
}

int cuda_rc(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return 0;
  std::snprintf(g_model_error, sizeof(g_model_error), "%s: %s (%d)", what, cudaGetErrorString(e), int(e));
  return int(e);
}

int blas_rc(cublasStatus_t s, const char* what) {
  if (s == CUBLAS_STATUS_SUCCESS) return 0;
  std::snprintf(g_model_error, sizeof(g_model_error), "%s: cuBLAS status %d", what, int(s));
  return 10000 + int(s);
}

int nvb_rc(int rc, const char* what) {
  if (rc == 0) return 0;
  std::snprintf(g_model_error, sizeof(g_model_error), "%s: %s", what, nvb_last_error());
  return rc;
}

#define TRY(expr)               \
  do {                          \
    if (int rc_ = (expr)) return rc_; \
  } while (0)

}  // namespace

struct NvbeModel {
  NvbeModelConfig c{};
  NvbeModelOptions o{};
  // weights (borrowed)
  const void* embedding = nullptr;
  const void* final_norm = nullptr;
  const void* lm_head = nullptr;
  std::vector<const void*> input_norm, qkv_w, q_norm, k_norm, o_proj, post_norm, gate_up_w, down_w;
  // owned device memory
  std::vector<void*> owned;
  std::vector<void*> k_cache, v_cache;
  uint8_t* metadata = nullptr;
  int *tokens = nullptr, *positions = nullptr, *seq_ids = nullptr, *slots = nullptr, *tables = nullptr,
      *last_idx = nullptr, *cu_q = nullptr, *kv_lens = nullptr, *samples = nullptr, *part_index = nullptr;
  float *temps = nullptr, *rope = nullptr, *part_score = nullptr, *lse_accum = nullptr, *out_accum = nullptr;
  uint64_t* seeds = nullptr;
  void *residual = nullptr, *hidden = nullptr, *normed = nullptr, *qkv = nullptr, *query = nullptr,
       *attention = nullptr, *gate_up = nullptr, *activated = nullptr, *gathered = nullptr, *logits = nullptr;
  // host
  NvbhMetadataLayout layout{};
  uint8_t* staging = nullptr;   // pinned
  int32_t* samples_host = nullptr;  // pinned
  std::vector<int32_t> cu_q_host, kv_lens_host;
  std::vector<int> decode_splits;
  int table_stride = 0, sms = 0, max_splits = 1;
  cudaStream_t stream = nullptr;
  cublasHandle_t blas = nullptr;
  std::unordered_map<int, cudaGraphExec_t> graphs;
  size_t last_samples = 0;
  // tcgen05 decode GEMMs: weight maps per layer, input maps per row count.
  std::vector<CUtensorMap> map_qkv, map_o, map_gate_up, map_down;
  std::unordered_map<int, CUtensorMap> map_in[4];  // normed, attention, activated, gathered; keyed by rows
  CUtensorMap map_lm{};  // LM head weights for the fused LM head + sampler
  float* fused_score = nullptr;  // [max_sequences][tiles] per-tile bests of the fused sampler
  int* fused_index = nullptr;
  void* gemm_ws = nullptr;  // split-K partials of the decode GEMMs
  size_t gemm_ws_bytes = 0;

  int alloc(void** p, size_t bytes, const char* what) {
    TRY(cuda_rc(cudaMalloc(p, bytes), what));
    owned.push_back(*p);
    return cuda_rc(cudaMemsetAsync(*p, 0, bytes, stream), what);
  }
  int gemm(const void* x, const void* w, void* y, int m, int n, int k);
  int tc_gemm(int which, const CUtensorMap& wmap, void* y, int m, int n, int k, bool silu);
  int forward(int rows, int sequences, int samples, int max_q, int max_k);
  void release();
};

// Row-major Y[m, n] = X[m, k] W[n, k]^T as the column-major Y^T = W X^T,
// the same cublasGemmEx call as kernels/kernels.cu:98-106.
int NvbeModel::gemm(const void* x, const void* w, void* y, int m, int n, int k) {
  const float alpha = 1.0f, beta = 0.0f;
  return blas_rc(cublasGemmEx(blas, CUBLAS_OP_T, CUBLAS_OP_N, n, m, k, &alpha, w, CUDA_R_16BF, k, x, CUDA_R_16BF, k,
                              &beta, y, CUDA_R_16BF, n, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT),
                 "cublasGemmEx");
}

// The decode GEMM from input buffer `which` (0 normed, 1 attention, 2
// activated) with `m` rows; the input map is built once per row count.
int NvbeModel::tc_gemm(int which, const CUtensorMap& wmap, void* y, int m, int n, int k, bool silu) {
  auto it = map_in[which].find(m);
  if (it == map_in[which].end()) {
    const void* x = which == 0 ? normed : which == 1 ? attention : which == 2 ? activated : gathered;
    CUtensorMap map;
    if (nvbm::gemm_input_map(x, m, k, &map)) return mfail("decode GEMM input map (rows %d, K %d)", m, k);
    it = map_in[which].emplace(m, map).first;
  }
  return cuda_rc(nvbm::launch_gemm_decode(stream, wmap, it->second, y, m, n, k, silu ? n / 2 : n, silu, sms, gemm_ws,
                                          gemm_ws_bytes),
                 "decode GEMM launch");
}

void NvbeModel::release() {
  for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
  graphs.clear();
  if (stream) cudaStreamSynchronize(stream);
  for (void* p : owned) cudaFree(p);
  owned.clear();
  if (staging) cudaFreeHost(staging);
  if (samples_host) cudaFreeHost(samples_host);
  staging = nullptr;
  samples_host = nullptr;
  if (blas) cublasDestroy(blas);
  if (stream) cudaStreamDestroy(stream);
  blas = nullptr;
  stream = nullptr;
}

// src/model.rs:635-818, with the attention seam on this library's kernels.
int NvbeModel::forward(int rows, int sequences, int nsamples, int max_q, int max_k) {
  const int H = c.hidden_size, D = c.head_dim, qh = c.num_attention_heads, kvh = c.num_key_value_heads;
  const int q_size = qh * D, qkv_size = q_size + 2 * kvh * D, I = c.intermediate_size;
  TRY(cuda_rc(nvbm::launch_embedding(stream, tokens, embedding, residual, rows, H, c.vocab_size, sms), "embedding"));
  const int splits = max_q == 1 ? decode_splits[size_t(sequences)] : 1;
  // tcgen05 decode GEMMs where they beat cuBLAS (small batches); cuBLAS else.
  auto tc = [&](int n, int k) { return o.tc_gemms && nvbm::gemm_decode_preferred(rows, n, k); };
  for (int l = 0; l < c.num_hidden_layers; ++l) {
    if (l == 0)
      TRY(cuda_rc(nvbm::launch_rms(stream, residual, nullptr, input_norm[l], normed, rows, H, c.rms_norm_eps),
                  "rms_norm"));
    else
      TRY(cuda_rc(nvbm::launch_rms(stream, hidden, residual, input_norm[l], normed, rows, H, c.rms_norm_eps),
                  "add_rms_norm"));
    if (tc(qkv_size, H))
      TRY(tc_gemm(0, map_qkv[size_t(l)], qkv, rows, qkv_size, H, false));
    else
      TRY(gemm(normed, qkv_w[l], qkv, rows, qkv_size, H));
    TRY(nvb_rc(nvb_qkv_rope_cached(stream, qkv, q_norm[l], k_norm[l], positions, slots, query, k_cache[l],
                                   v_cache[l], rows, qh, kvh, D, o.block_size, o.num_blocks, c.rms_norm_eps, rope,
                                   o.max_model_len),
               "nvb_qkv_rope_cached"));
    TRY(nvb_rc(nvb_paged_fwd_ex(stream, query, k_cache[l], v_cache[l], attention, cu_q, kv_lens, tables, sequences,
                                rows, max_q, max_k, qh, kvh, o.block_size, table_stride, splits, nullptr,
                                splits > 1 ? lse_accum : nullptr, splits > 1 ? out_accum : nullptr, o.num_blocks),
               "nvb_paged_fwd_ex"));
    if (tc(H, q_size))
      TRY(tc_gemm(1, map_o[size_t(l)], hidden, rows, H, q_size, false));
    else
      TRY(gemm(attention, o_proj[l], hidden, rows, H, q_size));
    TRY(cuda_rc(nvbm::launch_rms(stream, hidden, residual, post_norm[l], normed, rows, H, c.rms_norm_eps),
                "add_rms_norm"));
    if (tc(2 * I, H)) {
      // gate/up projection with SiLU * up fused into its epilogue
      TRY(tc_gemm(0, map_gate_up[size_t(l)], activated, rows, 2 * I, H, true));
    } else {
      TRY(gemm(normed, gate_up_w[l], gate_up, rows, 2 * I, H));
      TRY(cuda_rc(nvbm::launch_silu_mul(stream, gate_up, activated, rows, I, sms), "silu_mul"));
    }
    if (tc(H, I))
      TRY(tc_gemm(2, map_down[size_t(l)], hidden, rows, H, I, false));
    else
      TRY(gemm(activated, down_w[l], hidden, rows, H, I));
  }
  if (nsamples > 0) {
    TRY(cuda_rc(nvbm::launch_rms(stream, hidden, residual, final_norm, normed, rows, H, c.rms_norm_eps),
                "final add_rms_norm"));
    TRY(cuda_rc(nvbm::launch_gather(stream, normed, last_idx, gathered, nsamples, H, rows, sms), "gather"));
    if (o.tc_gemms && nvbm::gemm_sample_preferred(nsamples)) {
      // LM head with the Gumbel-max sampler fused into its epilogue
      auto it = map_in[3].find(nsamples);
      if (it == map_in[3].end()) {
        CUtensorMap map;
        if (nvbm::gemm_input_map(gathered, nsamples, H, &map)) return mfail("LM head input map");
        it = map_in[3].emplace(nsamples, map).first;
      }
      TRY(cuda_rc(nvbm::launch_gemm_decode_sample(stream, map_lm, it->second, logits, nsamples, c.vocab_size, H,
                                                  temps, seeds, fused_score, fused_index),
                  "fused LM head + sampler"));
      TRY(cuda_rc(nvbm::launch_sample_combine(stream, fused_score, fused_index, samples, nsamples,
                                              nvbm::gemm_decode_tiles(c.vocab_size)),
                  "sample combine"));
    } else {
      TRY(gemm(gathered, lm_head ? lm_head : embedding, logits, nsamples, c.vocab_size, H));
      TRY(cuda_rc(nvbm::launch_sample(stream, logits, temps, seeds, samples, part_score, part_index, nsamples,
                                      c.vocab_size),
                  "sample"));
    }
  }
  return 0;
}

namespace {

int create_impl(NvbeModel* m, const NvbeModelConfig* cfg, const NvbeModelOptions* opt, const NvbeModelWeights* w) {
  const NvbeModelConfig& c = *cfg;
  const NvbeModelOptions& o = *opt;
  // Capacity checks of QwenModel::load (src/model.rs:381-412) for this path.
  if (c.hidden_size <= 0 || c.intermediate_size <= 0 || c.num_hidden_layers <= 0 || c.vocab_size <= 0 ||
      c.num_attention_heads <= 0 || c.num_key_value_heads <= 0 || c.num_attention_heads % c.num_key_value_heads)
    return mfail("model dimensions must be positive and query heads a multiple of KV heads");
  if (c.head_dim != 128) return mfail("the paged attention kernels need head_dim 128 (got %d)", c.head_dim);
  if (c.hidden_size % 8 || c.intermediate_size % 8) return mfail("hidden and intermediate sizes must be multiples of 8");
  if (!(c.rms_norm_eps > 0.0f) || !(c.rope_theta > 0.0f)) return mfail("RMS epsilon and RoPE theta must be positive");
  if (o.block_size <= 0 || o.num_blocks <= 0 || o.max_batch_tokens <= 0 || o.max_sequences <= 0 ||
      o.max_model_len <= 0)
    return mfail("all model capacities must be positive");
  if (o.block_size % 256) return mfail("block_size must be a multiple of 256");
  if (o.max_sequences > o.max_batch_tokens) return mfail("max_sequences must not exceed max_batch_tokens");
  if ((long long)o.num_blocks * o.block_size > 0x7fffffffLL) return mfail("configured capacity exceeds 32-bit CUDA indexing");
  if (o.max_sequences > 65535) return mfail("max_sequences must be at most 65535");
  if (!w || !w->embedding || !w->final_norm || !w->input_norm || !w->qkv || !w->q_norm || !w->k_norm || !w->o_proj ||
      !w->post_norm || !w->gate_up || !w->down || (!c.tie_word_embeddings && !w->lm_head))
    return mfail("missing weights");
  m->c = c;
  m->o = o;
  const int L = c.num_hidden_layers;
  m->embedding = w->embedding;
  m->final_norm = w->final_norm;
  m->lm_head = c.tie_word_embeddings ? nullptr : w->lm_head;
  m->input_norm.assign(w->input_norm, w->input_norm + L);
  m->qkv_w.assign(w->qkv, w->qkv + L);
  m->q_norm.assign(w->q_norm, w->q_norm + L);
  m->k_norm.assign(w->k_norm, w->k_norm + L);
  m->o_proj.assign(w->o_proj, w->o_proj + L);
  m->post_norm.assign(w->post_norm, w->post_norm + L);
  m->gate_up_w.assign(w->gate_up, w->gate_up + L);
  m->down_w.assign(w->down, w->down + L);

  TRY(cuda_rc(cudaSetDevice(o.device), "cudaSetDevice"));
  TRY(cuda_rc(cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, o.device), "SM count"));
  TRY(cuda_rc(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking), "cudaStreamCreate"));
  TRY(blas_rc(cublasCreate(&m->blas), "cublasCreate"));
  TRY(blas_rc(cublasSetStream(m->blas, m->stream), "cublasSetStream"));

  m->table_stride = (o.max_model_len + o.block_size - 1) / o.block_size;
  const int T = o.max_batch_tokens, S = o.max_sequences, H = c.hidden_size, D = c.head_dim;
  const int qh = c.num_attention_heads, kvh = c.num_key_value_heads, I = c.intermediate_size;
  if (nvbh_metadata_layout(size_t(T), size_t(S), size_t(m->table_stride), &m->layout))
    return mfail("metadata layout: %s", nvbh_last_error());
  // Decode split counts per batch size with the geometry fixed by
  // max_model_len, so captured graphs stay valid as contexts grow
  // (src/model.rs:414-439, 947-949).
  m->decode_splits.assign(size_t(S) + 1, 1);
  for (int b = 1; b <= S; ++b) {
    const int s = nvb_num_splits(b, qh, kvh, o.max_model_len, m->sms);
    m->decode_splits[size_t(b)] = s < 1 ? 1 : s;
    m->max_splits = std::max(m->max_splits, m->decode_splits[size_t(b)]);
  }
  void* p = nullptr;
  TRY(m->alloc(&p, m->layout.bytes, "metadata"));
  m->metadata = static_cast<uint8_t*>(p);
  auto field = [&](int f) { return m->metadata + m->layout.start[f]; };
  m->tokens = reinterpret_cast<int*>(field(NVBH_META_TOKENS));
  m->positions = reinterpret_cast<int*>(field(NVBH_META_POSITIONS));
  m->seq_ids = reinterpret_cast<int*>(field(NVBH_META_SEQUENCES));
  m->slots = reinterpret_cast<int*>(field(NVBH_META_SLOTS));
  m->tables = reinterpret_cast<int*>(field(NVBH_META_TABLES));
  m->last_idx = reinterpret_cast<int*>(field(NVBH_META_LAST_INDICES));
  m->temps = reinterpret_cast<float*>(field(NVBH_META_TEMPERATURES));
  m->seeds = reinterpret_cast<uint64_t*>(field(NVBH_META_SEEDS));
  m->cu_q = reinterpret_cast<int*>(field(NVBH_META_CU_Q));
  m->kv_lens = reinterpret_cast<int*>(field(NVBH_META_KV_LENS));
  const size_t bf = 2;
  const int parts = nvbm::sample_partitions(c.vocab_size);
  struct Buf { void** dst; size_t bytes; const char* name; };
  const Buf bufs[] = {
      {&m->residual, size_t(T) * H * bf, "residual"}, {&m->hidden, size_t(T) * H * bf, "hidden"},
      {&m->normed, size_t(T) * H * bf, "normed"}, {&m->qkv, size_t(T) * (qh + 2 * kvh) * D * bf, "qkv"},
      {&m->query, size_t(T) * qh * D * bf, "query"}, {&m->attention, size_t(T) * qh * D * bf, "attention"},
      {&m->gate_up, size_t(T) * 2 * I * bf, "gate_up"}, {&m->activated, size_t(T) * I * bf, "activated"},
      {&m->gathered, size_t(S) * H * bf, "gathered"}, {&m->logits, size_t(S) * c.vocab_size * bf, "logits"},
      {reinterpret_cast<void**>(&m->samples), size_t(S) * 4, "samples"},
      {reinterpret_cast<void**>(&m->part_score), size_t(S) * parts * 4, "sample partials"},
      {reinterpret_cast<void**>(&m->part_index), size_t(S) * parts * 4, "sample partials"},
      {reinterpret_cast<void**>(&m->rope), size_t(o.max_model_len) * D * 4, "rope table"},
      {reinterpret_cast<void**>(&m->lse_accum), size_t(m->max_splits) * S * qh * 4, "split-KV lse"},
      {reinterpret_cast<void**>(&m->out_accum), size_t(m->max_splits) * S * qh * D * 4, "split-KV partials"},
  };
  for (const Buf& b : bufs) TRY(m->alloc(b.dst, b.bytes, b.name));
  const size_t cache_bytes = size_t(o.num_blocks) * o.block_size * kvh * D * bf;
  m->k_cache.resize(size_t(L));
  m->v_cache.resize(size_t(L));
  for (int l = 0; l < L; ++l) {
    TRY(m->alloc(&m->k_cache[size_t(l)], cache_bytes, "paged K cache; reduce num_blocks"));
    TRY(m->alloc(&m->v_cache[size_t(l)], cache_bytes, "paged V cache; reduce num_blocks"));
  }
  TRY(cuda_rc(cudaHostAlloc(reinterpret_cast<void**>(&m->staging), m->layout.bytes, cudaHostAllocDefault),
              "pinned metadata staging"));
  std::memset(m->staging, 0, m->layout.bytes);
  TRY(cuda_rc(cudaHostAlloc(reinterpret_cast<void**>(&m->samples_host), size_t(S) * 4, cudaHostAllocDefault),
              "pinned sample buffer"));
  m->cu_q_host.resize(size_t(S) + 1);
  m->kv_lens_host.resize(size_t(S));
  if (o.tc_gemms) {
    if (H % 64 || (qh * D) % 64 || I % 64 || (qh + 2 * kvh) * D % 8 || I % 8)
      return mfail("the tcgen05 GEMMs need hidden, attention and intermediate sizes that are multiples of 64");
    const int mmax = std::min(nvbm::gemm_decode_max_rows(), T);
    for (const auto& g : {std::array<int, 3>{(qh + 2 * kvh) * D, H, 0}, std::array<int, 3>{H, qh * D, 0},
                          std::array<int, 3>{2 * I, H, 1}, std::array<int, 3>{H, I, 0}})
      m->gemm_ws_bytes = std::max(m->gemm_ws_bytes, nvbm::gemm_decode_workspace(mmax, g[0], g[1], g[2] != 0, m->sms));
    TRY(m->alloc(&m->gemm_ws, m->gemm_ws_bytes, "decode GEMM workspace"));
    const size_t fused_parts = size_t(S) * size_t(nvbm::gemm_decode_tiles(c.vocab_size));
    void* fp = nullptr;
    TRY(m->alloc(&fp, fused_parts * 4, "fused sampler partials"));
    m->fused_score = static_cast<float*>(fp);
    TRY(m->alloc(&fp, fused_parts * 4, "fused sampler partials"));
    m->fused_index = static_cast<int*>(fp);
    if (c.vocab_size % 4 ||
        nvbm::gemm_weight_map(m->lm_head ? m->lm_head : m->embedding, c.vocab_size, H, false, &m->map_lm))
      return mfail("LM head tensor map (vocab a multiple of 4, 16-byte aligned weights)");
    m->map_qkv.resize(size_t(L));
    m->map_o.resize(size_t(L));
    m->map_gate_up.resize(size_t(L));
    m->map_down.resize(size_t(L));
    for (int l = 0; l < L; ++l) {
      const size_t i = size_t(l);
      if (nvbm::gemm_weight_map(m->qkv_w[i], (qh + 2 * kvh) * D, H, false, &m->map_qkv[i]) ||
          nvbm::gemm_weight_map(m->o_proj[i], H, qh * D, false, &m->map_o[i]) ||
          nvbm::gemm_weight_map(m->gate_up_w[i], 2 * I, H, true, &m->map_gate_up[i]) ||
          nvbm::gemm_weight_map(m->down_w[i], H, I, false, &m->map_down[i]))
        return mfail("tensor maps of layer %d's weights (16-byte aligned BF16 [out, in] expected)", l);
    }
  }
  TRY(nvb_rc(nvb_rope_cache(m->stream, m->rope, o.max_model_len, D, c.rope_theta), "nvb_rope_cache"));
  return cuda_rc(cudaStreamSynchronize(m->stream), "model load synchronize");
}

}  // namespace

extern "C" {

const char* nvbe_model_last_error(void) { return g_model_error; }

int nvbe_model_create(const NvbeModelConfig* config, const NvbeModelOptions* options,
                      const NvbeModelWeights* weights, NvbeModel** out) {
  g_model_error[0] = 0;
  if (!config || !options || !out) return mfail("null model argument");
  NvbeModel* m = new (std::nothrow) NvbeModel();
  if (!m) return mfail("host allocation failed");
  const int rc = create_impl(m, config, options, weights);
  if (rc) {
    m->release();
    delete m;
    return rc;
  }
  *out = m;
  return 0;
}

void nvbe_model_destroy(NvbeModel* m) {
  if (!m) return;
  cudaSetDevice(m->o.device);
  m->release();
  delete m;
}

int nvbe_model_sync(void* model) {
  NvbeModel* m = static_cast<NvbeModel*>(model);
  if (!m) return mfail("null model");
  return cuda_rc(cudaStreamSynchronize(m->stream), "cudaStreamSynchronize");
}

int nvbe_model_run(void* model, const NvbhBatch* batch, uint32_t* sampled) {
  g_model_error[0] = 0;
  NvbeModel* m = static_cast<NvbeModel*>(model);
  if (!m || !batch || (batch->samples && !sampled)) return mfail("null run argument");
  TRY(cuda_rc(cudaSetDevice(m->o.device), "cudaSetDevice"));
  const NvbhLimits lim{size_t(m->o.max_batch_tokens), size_t(m->o.max_sequences), size_t(m->o.max_model_len),
                       size_t(m->o.block_size),       size_t(m->o.num_blocks),    size_t(m->table_stride),
                       size_t(m->c.vocab_size)};
  size_t rows = 0, sequences = 0, nsamples = 0, max_q = 0;
  if (nvbh_validate_batch(batch, &lim, &rows, &sequences, &nsamples)) return mfail("%s", nvbh_last_error());
  m->last_samples = 0;
  if (nvbh_flash_metadata(batch->positions, batch->sequence_ids, rows, sequences, m->cu_q_host.data(),
                          m->kv_lens_host.data(), &max_q))
    return mfail("%s", nvbh_last_error());
  // Decode geometry is fixed by max_model_len so a captured graph stays
  // valid as contexts grow; prefill uses the longest context.
  int max_k = m->o.max_model_len;
  if (max_q != 1) max_k = *std::max_element(m->kv_lens_host.begin(), m->kv_lens_host.begin() + long(sequences));
  if (nvbh_metadata_pack(&m->layout, m->staging, m->layout.bytes, batch, sequences, size_t(m->table_stride),
                         m->cu_q_host.data(), m->kv_lens_host.data()))
    return mfail("%s", nvbh_last_error());
  TRY(cuda_rc(cudaMemcpyAsync(m->metadata, m->staging, m->layout.bytes, cudaMemcpyHostToDevice, m->stream),
              "metadata upload"));
  const int r = int(rows), s = int(sequences), k = int(nsamples), q = int(max_q);
  if (m->o.cuda_graphs && batch->is_decode && rows == sequences && nsamples == sequences) {
    auto it = m->graphs.find(r);
    if (it == m->graphs.end()) {
      // Warm-up forward first (cuBLAS initialises per-shape state, the
      // attention library encodes its TMA descriptors), then capture; the
      // replay below rewrites the same KV slots with the same values.
      TRY(m->forward(r, s, k, q, max_k));
      TRY(cuda_rc(cudaStreamSynchronize(m->stream), "warm-up synchronize"));
      TRY(cuda_rc(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture"));
      const int frc = m->forward(r, s, k, q, max_k);
      cudaGraph_t graph = nullptr;
      const cudaError_t end = cudaStreamEndCapture(m->stream, &graph);
      if (frc) {
        if (graph) cudaGraphDestroy(graph);
        return frc;
      }
      TRY(cuda_rc(end, "cudaStreamEndCapture"));
      cudaGraphExec_t exec = nullptr;
      const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
      cudaGraphDestroy(graph);
      TRY(cuda_rc(inst, "cudaGraphInstantiate"));
      it = m->graphs.emplace(r, exec).first;
    }
    TRY(cuda_rc(cudaGraphLaunch(it->second, m->stream), "cudaGraphLaunch"));
  } else {
    TRY(m->forward(r, s, k, q, max_k));
  }
  if (k > 0)
    TRY(cuda_rc(cudaMemcpyAsync(m->samples_host, m->samples, size_t(k) * 4, cudaMemcpyDeviceToHost, m->stream),
                "sample download"));
  TRY(cuda_rc(cudaStreamSynchronize(m->stream), "step synchronize"));
  for (int i = 0; i < k; ++i) {
    const int32_t id = m->samples_host[i];
    if (id < 0 || id >= m->c.vocab_size) return mfail("GPU sampler returned an invalid token id");
    sampled[i] = uint32_t(id);
  }
  m->last_samples = size_t(k);
  return 0;
}

int nvbe_model_last_logits(NvbeModel* m, uint16_t* out, size_t capacity, size_t* samples) {
  g_model_error[0] = 0;
  if (!m || !samples) return mfail("null argument");
  *samples = m->last_samples;
  const size_t n = m->last_samples * size_t(m->c.vocab_size);
  if (!n) return 0;
  if (!out || capacity < n) return mfail("logit buffer holds %zu values, needs %zu", capacity, n);
  return cuda_rc(cudaMemcpy(out, m->logits, n * 2, cudaMemcpyDeviceToHost), "logit download");
}

int nvbe_model_kv_cache(NvbeModel* m, int layer, void** k, void** v) {
  if (!m || layer < 0 || layer >= m->c.num_hidden_layers || !k || !v) return mfail("invalid layer");
  *k = m->k_cache[size_t(layer)];
  *v = m->v_cache[size_t(layer)];
  return 0;
}

void* nvbe_model_stream(NvbeModel* m) { return m ? static_cast<void*>(m->stream) : nullptr; }

size_t nvbe_model_graph_count(const NvbeModel* m) { return m ? m->graphs.size() : 0; }

}  // extern "C"

// ------------------------------------------------------------ layer kernels
// Stream-based replacements of the reference's per-layer entry points
// (kernels/kernels.cu:470-500, whose first argument is its Context*).
namespace {

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev))
    return 148;
  return n > 0 ? n : 148;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int nvbe_layer_embedding(void* stream, const int* tokens, const void* weight, void* out, int rows, int hidden,
                         int vocab) {
  g_model_error[0] = 0;
  if (!tokens || !weight || !out || rows <= 0 || hidden <= 0 || hidden % 8 || vocab <= 0 || !aligned16(weight) ||
      !aligned16(out))
    return mfail("invalid embedding arguments");
  return cuda_rc(nvbm::launch_embedding(static_cast<cudaStream_t>(stream), tokens, weight, out, rows, hidden, vocab,
                                        sm_count()),
                 "embedding launch");
}

int nvbe_layer_rms(void* stream, const void* x, const void* weight, void* out, int rows, int hidden, float eps) {
  g_model_error[0] = 0;
  if (!x || !weight || !out || rows <= 0 || hidden <= 0 || !(eps >= 0.0f)) return mfail("invalid rms arguments");
  return cuda_rc(nvbm::launch_rms(static_cast<cudaStream_t>(stream), x, nullptr, weight, out, rows, hidden, eps),
                 "rms launch");
}

int nvbe_layer_add_rms(void* stream, const void* x, void* residual, const void* weight, void* out, int rows,
                       int hidden, float eps) {
  g_model_error[0] = 0;
  if (!x || !residual || !weight || !out || rows <= 0 || hidden <= 0 || !(eps >= 0.0f))
    return mfail("invalid add_rms arguments");
  return cuda_rc(nvbm::launch_rms(static_cast<cudaStream_t>(stream), x, residual, weight, out, rows, hidden, eps),
                 "add_rms launch");
}

int nvbe_layer_silu_mul(void* stream, const void* packed, void* out, int rows, int intermediate) {
  g_model_error[0] = 0;
  if (!packed || !out || rows <= 0 || intermediate <= 0 || intermediate % 8 || !aligned16(packed) || !aligned16(out))
    return mfail("invalid silu arguments");
  return cuda_rc(nvbm::launch_silu_mul(static_cast<cudaStream_t>(stream), packed, out, rows, intermediate, sm_count()),
                 "silu launch");
}

int nvbe_layer_gather(void* stream, const void* x, const int* indices, void* out, int rows, int hidden,
                      int input_rows) {
  g_model_error[0] = 0;
  if (!x || !indices || !out || rows <= 0 || hidden <= 0 || hidden % 8 || input_rows <= 0 || !aligned16(x) ||
      !aligned16(out))
    return mfail("invalid gather arguments");
  return cuda_rc(nvbm::launch_gather(static_cast<cudaStream_t>(stream), x, indices, out, rows, hidden, input_rows,
                                     sm_count()),
                 "gather launch");
}

size_t nvbe_gemm_workspace_bytes(int M, int N, int K, int silu) {
  if (M < 1 || M > nvbm::gemm_decode_max_rows() || N < 4 || K < 64) return 0;
  return nvbm::gemm_decode_workspace(M, N, K, silu != 0, sm_count());
}

int nvbe_layer_gemm(void* stream, const void* x, const void* w, void* y, int M, int N, int K, int silu,
                    void* workspace, size_t workspace_bytes) {
  g_model_error[0] = 0;
  if (!x || !w || !y || M < 1 || M > nvbm::gemm_decode_max_rows() || N < 4 || N % (silu ? 8 : 4) || K < 64 ||
      K % 64 || !aligned16(x) || !aligned16(w) || !aligned16(y))
    return mfail("invalid decode GEMM arguments (M in [1, 256], K a multiple of 64, N of 4 or 8 with silu)");
  const size_t need = nvbm::gemm_decode_workspace(M, N, K, silu != 0, sm_count());
  if (!workspace || !aligned16(workspace) || workspace_bytes < need)
    return mfail("the decode GEMM needs a 16-byte aligned workspace of %zu bytes (got %zu)", need, workspace_bytes);
  CUtensorMap wmap, xmap;
  if (nvbm::gemm_weight_map(w, N, K, silu != 0, &wmap) || nvbm::gemm_input_map(x, M, K, &xmap))
    return mfail("decode GEMM tensor maps");
  return cuda_rc(nvbm::launch_gemm_decode(static_cast<cudaStream_t>(stream), wmap, xmap, y, M, N, K,
                                          silu ? N / 2 : N, silu != 0, sm_count(), workspace, workspace_bytes),
                 "decode GEMM launch");
}

int nvbe_gemm_device_error(void) { return nvbm::gemm_decode_error(); }

int nvbe_gemm_sample_tiles(int vocab) { return vocab > 0 ? nvbm::gemm_decode_tiles(vocab) : 0; }

int nvbe_layer_gemm_sample(void* stream, const void* x, const void* w, void* logits, int M, int N, int K,
                           const float* temperatures, const uint64_t* seeds, int* out, float* partial_scores,
                           int* partial_indices) {
  g_model_error[0] = 0;
  if (!x || !w || !logits || !temperatures || !seeds || !out || !partial_scores || !partial_indices || M < 1 ||
      M > nvbm::gemm_decode_max_rows() || N < 4 || N % 4 || K < 64 || K % 64 || !aligned16(x) || !aligned16(w) ||
      !aligned16(logits))
    return mfail("invalid fused LM head arguments (M in [1, 256], K a multiple of 64, N of 4)");
  CUtensorMap wmap, xmap;
  if (nvbm::gemm_weight_map(w, N, K, false, &wmap) || nvbm::gemm_input_map(x, M, K, &xmap))
    return mfail("fused LM head tensor maps");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = cuda_rc(nvbm::launch_gemm_decode_sample(s, wmap, xmap, logits, M, N, K, temperatures, seeds,
                                                   partial_scores, partial_indices),
                   "fused LM head launch");
  if (rc) return rc;
  return cuda_rc(nvbm::launch_sample_combine(s, partial_scores, partial_indices, out, M, nvbm::gemm_decode_tiles(N)),
                 "sample combine launch");
}

int nvbe_sample_partitions(int vocab) { return vocab > 0 ? nvbm::sample_partitions(vocab) : 0; }

int nvbe_layer_sample(void* stream, const void* logits, const float* temperatures, const uint64_t* seeds, int* out,
                      float* partial_scores, int* partial_indices, int rows, int vocab) {
  g_model_error[0] = 0;
  if (!logits || !temperatures || !seeds || !out || !partial_scores || !partial_indices || rows <= 0 ||
      rows > 65535 || vocab <= 0)
    return mfail("invalid sample arguments");
  return cuda_rc(nvbm::launch_sample(static_cast<cudaStream_t>(stream), logits, temperatures, seeds, out,
                                     partial_scores, partial_indices, rows, vocab),
                 "sample launch");
}

}  // extern "C"
