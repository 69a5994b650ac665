// Continuous-batching scheduler (include/nvb_engine.h, nvbe_engine_*).
//
// Restates the reference's LlmEngine (src/runtime.rs:358-777) in C++ on top
// of this library's page pool and batch builder (runtime.cpp):
//   admission            src/runtime.rs:462-512 (pages for the retained
//                        prompt, minus live shared prefix pages)
//   step loop            src/runtime.rs:514-688 (prefill and decode in
//                        separate forwards, chunked prefill under
//                        max_batch_tokens, preemption of the youngest
//                        sequence not in the batch, prefix publication)
//   request validation   src/runtime.rs:411-455
// The model is reached through NvbeRunFn, so the same scheduler drives the
// GPU runner (libnvb_model.so) and the CPU test runners.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <deque>
#include <limits>
#include <new>
#include <unordered_set>
#include <vector>

#include "nvb_engine.h"

namespace {

thread_local char g_engine_error[512] = {};

int efail(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  std::vsnprintf(g_engine_error, sizeof(g_engine_error), fmt, args);
  va_end(args);
  return -1;
}

constexpr size_t kI32Max = size_t(std::numeric_limits<int32_t>::max());

enum class Status { Waiting, Active, Finished };

struct Sequence {
  const NvbeRequest* request = nullptr;
  std::vector<uint32_t> tokens;
  size_t computed = 0;
  std::vector<int32_t> blocks;
  Status status = Status::Waiting;
  size_t cached_tokens = 0;
  double first_token_ms = -1.0;
  double previous_token_ms = -1.0;
  double latency_ms = 0.0;
  std::vector<double> gaps_ms;
  int finish_reason = NVBE_FINISH_LENGTH;

  size_t generated() const { return tokens.size() - request->prompt_len; }
  bool is_decode() const { return generated() > 0 && computed + 1 == tokens.size(); }
  void release(NvbhBlockPool* pool) {
    for (int32_t b : blocks) nvbh_pool_release(pool, b);
    blocks.clear();
    computed = 0;
  }
};

struct Segment {
  size_t sequence, start, end;
  bool sample;
};

size_t ceil_div(size_t a, size_t b) { return (a + b - 1) / b; }

}  // namespace

struct NvbeEngine {
  NvbeSchedulerConfig config{};
  NvbeRunFn run = nullptr;
  NvbeSyncFn sync = nullptr;
  void* runner = nullptr;
  NvbhBlockPool* pool = nullptr;
  bool failed = false;
  // make_batch output buffers, sized once from the configuration.
  std::vector<int32_t> token_ids, positions, sequence_ids, slot_mapping, block_tables, last_token_indices;
  std::vector<float> temperatures;
  std::vector<uint64_t> seeds;
  std::vector<uint32_t> sampled;

  int synchronize() {
    if (!sync) return 0;
    const int rc = sync(runner);
    return rc ? efail("model runner synchronize failed (status %d)", rc) : 0;
  }
  int validate_requests(const NvbeRequest* requests, size_t n) const;
  size_t admission_blocks(const Sequence& s) const;
  int admit(Sequence& s, NvbeRunStats& stats);
  int execute(std::vector<Sequence>& seqs, uint64_t seed, NvbeRunStats& stats,
              std::chrono::steady_clock::time_point started);
};

extern "C" int nvbe_scheduler_config_validate(const NvbeSchedulerConfig* c) {
  g_engine_error[0] = 0;
  if (!c) return efail("null scheduler config");
  if (c->block_size == 0) return efail("block_size must be positive");
  if (c->num_blocks == 0) return efail("num_blocks must be positive");
  if (c->max_sequences == 0) return efail("max_sequences must be positive");
  if (c->max_model_len == 0) return efail("max_model_len must be positive");
  if (c->max_batch_tokens == 0) return efail("max_batch_tokens must be positive");
  if (c->num_blocks > kI32Max / c->block_size) return efail("KV slot indices must fit in i32");
  if (c->max_model_len > kI32Max || c->max_sequences > kI32Max || c->max_batch_tokens > kI32Max)
    return efail("batch dimensions must fit in i32");
  return 0;
}

int NvbeEngine::validate_requests(const NvbeRequest* requests, size_t n) const {
  std::unordered_set<uint64_t> ids;
  for (size_t i = 0; i < n; ++i) {
    const NvbeRequest& r = requests[i];
    if (!ids.insert(r.id).second) return efail("duplicate request ID %llu", (unsigned long long)r.id);
    if (r.prompt_len == 0 || !r.prompt_token_ids) return efail("prompt must not be empty");
    if (r.max_tokens == 0) return efail("max_tokens must be positive");
    if (!std::isfinite(r.temperature) || r.temperature < 0.0f)
      return efail("temperature must be finite and nonnegative");
    for (size_t t = 0; t < r.prompt_len; ++t)
      if (r.prompt_token_ids[t] > uint32_t(kI32Max)) return efail("token IDs must fit in i32");
    if (r.max_tokens > std::numeric_limits<size_t>::max() - r.prompt_len) return efail("request token length overflow");
    const size_t length = r.prompt_len + r.max_tokens;
    if (length > config.max_model_len)
      return efail("request %llu needs %zu context tokens, exceeding max_model_len %zu", (unsigned long long)r.id,
                   length, config.max_model_len);
    // The final sampled token is returned without a further KV write.
    const size_t needed = ceil_div(length - 1, config.block_size);
    if (needed > config.num_blocks)
      return efail("request %llu needs up to %zu KV blocks but only %zu exist", (unsigned long long)r.id, needed,
                   config.num_blocks);
  }
  return 0;
}

// Pages needed to compute the retained tokens (src/runtime.rs:457-475):
// already-pinned matching prefix pages cost nothing new, while unreferenced
// cached pages still have to come out of the free pool.
size_t NvbeEngine::admission_blocks(const Sequence& s) const {
  size_t needed = ceil_div(s.tokens.size(), config.block_size);
  if (config.prefix_caching) {
    const size_t reusable = (s.tokens.size() - 1) / config.block_size;
    for (size_t logical = 0; logical < reusable; ++logical) {
      const int block = nvbh_pool_find(pool, s.tokens.data(), (logical + 1) * config.block_size);
      if (block < 0) break;
      if (nvbh_pool_references(pool, block) > 0) --needed;
    }
  }
  return needed;
}

// src/runtime.rs:477-512: retain cached prefix pages, then reserve this
// prefill's pages. At least the final prompt token is always recomputed.
int NvbeEngine::admit(Sequence& s, NvbeRunStats& stats) {
  s.status = Status::Active;
  const size_t bs = config.block_size;
  const size_t reusable = config.prefix_caching ? (s.tokens.size() - 1) / bs : 0;
  for (size_t logical = 0; logical < reusable; ++logical) {
    const size_t end = (logical + 1) * bs;
    const int block = nvbh_pool_find_and_retain(pool, s.tokens.data(), end);
    if (block < 0) break;
    s.blocks.push_back(block);
    s.computed = end;
    s.cached_tokens += bs;
    stats.cached_tokens += bs;
    stats.cache_hits += 1;
  }
  while (s.blocks.size() < ceil_div(s.tokens.size(), bs)) {
    const int block = nvbh_pool_allocate(pool);
    if (block < 0) return efail("prefill admission capacity invariant violated");
    s.blocks.push_back(block);
  }
  const size_t in_use = nvbh_pool_in_use(pool);
  if (in_use > stats.peak_kv_blocks) stats.peak_kv_blocks = in_use;
  return 0;
}

int NvbeEngine::execute(std::vector<Sequence>& seqs, uint64_t seed, NvbeRunStats& stats,
                        std::chrono::steady_clock::time_point started) {
  using clock = std::chrono::steady_clock;
  const size_t bs = config.block_size;
  std::deque<size_t> waiting;
  for (size_t i = 0; i < seqs.size(); ++i) waiting.push_back(i);
  std::vector<size_t> active, candidates;
  std::vector<Segment> segments;
  std::vector<NvbhSegment> nsegs;
  size_t finished = 0;
  for (const auto& s : seqs) stats.input_tokens += s.tokens.size();
  stats.total_requests = seqs.size();

  while (finished < seqs.size()) {
    while (active.size() < config.max_sequences && !waiting.empty()) {
      const size_t index = waiting.front();
      const size_t needed = admission_blocks(seqs[index]);
      // Pages the next decode step of the running sequences needs stay protected.
      size_t decode_growth = 0;
      for (size_t i : active) {
        const size_t want = ceil_div(seqs[i].tokens.size(), bs);
        decode_growth += want > seqs[i].blocks.size() ? want - seqs[i].blocks.size() : 0;
      }
      if (needed + decode_growth > nvbh_pool_available(pool)) break;
      waiting.pop_front();
      if (int rc = admit(seqs[index], stats)) return rc;
      active.push_back(index);
    }
    if (active.empty()) return efail("scheduler made no progress");

    // Prefill and decode run as separate forwards; prefill is chunked by the
    // token budget (src/runtime.rs:557-565). With mixed_batches, decode rows
    // come first and prefill chunks fill the rest of the budget.
    bool is_decode = true;
    for (size_t i : active) is_decode = is_decode && seqs[i].is_decode();
    candidates.clear();
    if (config.mixed_batches) {
      for (size_t i : active)
        if (seqs[i].is_decode()) candidates.push_back(i);
      for (size_t i : active)
        if (!seqs[i].is_decode()) candidates.push_back(i);
    } else {
      for (size_t i : active)
        if (seqs[i].is_decode() == is_decode) candidates.push_back(i);
    }
    if (is_decode) {
      // Longest context first: the attention kernels claim (sequence, kv
      // head) items in row order, so a step ends on short items instead of
      // a long one started last. Rows are independent, so the order changes
      // no result.
      std::stable_sort(candidates.begin(), candidates.end(), [&](size_t a, size_t b) {
        return seqs[a].tokens.size() > seqs[b].tokens.size();
      });
    }
    segments.clear();
    size_t budget = config.max_batch_tokens;
    for (size_t index : candidates) {
      Sequence& s = seqs[index];
      if (budget == 0 || s.status != Status::Active) continue;
      const size_t start = s.computed;
      size_t end = std::min(s.tokens.size(), start + budget);
      const size_t desired = ceil_div(end, bs);
      const size_t extra = desired > s.blocks.size() ? desired - s.blocks.size() : 0;
      while (nvbh_pool_available(pool) < extra) {
        // Rows already in this batch stay pinned; preempt the youngest other
        // sequence holding pages (src/runtime.rs:583-602).
        long victim = -1;
        for (size_t k = active.size(); k-- > 0;) {
          const size_t other = active[k];
          if (other == index || seqs[other].blocks.empty()) continue;
          bool in_batch = false;
          for (const auto& seg : segments) in_batch = in_batch || seg.sequence == other;
          if (in_batch) continue;
          victim = long(other);
          break;
        }
        if (victim < 0) break;
        seqs[size_t(victim)].release(pool);
        seqs[size_t(victim)].status = Status::Waiting;
        for (size_t k = 0; k < active.size(); ++k)
          if (active[k] == size_t(victim)) {
            active.erase(active.begin() + long(k));
            break;
          }
        waiting.push_front(size_t(victim));
        stats.preemptions += 1;
      }
      const size_t capacity = (s.blocks.size() + nvbh_pool_available(pool)) * bs;
      end = std::min(end, capacity);
      if (end <= start) continue;
      while (s.blocks.size() < ceil_div(end, bs)) {
        const int block = nvbh_pool_allocate(pool);
        if (block < 0) return efail("KV allocation invariant violated");
        s.blocks.push_back(block);
      }
      const size_t in_use = nvbh_pool_in_use(pool);
      if (in_use > stats.peak_kv_blocks) stats.peak_kv_blocks = in_use;
      segments.push_back({index, start, end, end == s.tokens.size()});
      budget -= end - start;
    }
    if (segments.empty()) return efail("KV pressure prevented scheduler progress");

    // make_batch (src/runtime.rs:728-777) through runtime.cpp.
    nsegs.resize(segments.size());
    for (size_t k = 0; k < segments.size(); ++k) {
      const Sequence& s = seqs[segments[k].sequence];
      NvbhSegment& g = nsegs[k];
      g.tokens = s.tokens.data();
      g.num_tokens = s.tokens.size();
      g.blocks = s.blocks.data();
      g.num_blocks = s.blocks.size();
      g.start = segments[k].start;
      g.end = segments[k].end;
      g.sample = segments[k].sample ? 1 : 0;
      g.request_id = s.request->id;
      g.generated = s.generated();
      g.temperature = s.request->temperature;
    }
    NvbhBatchOut out{};
    out.token_ids = token_ids.data();
    out.positions = positions.data();
    out.sequence_ids = sequence_ids.data();
    out.slot_mapping = slot_mapping.data();
    out.rows_cap = token_ids.size();
    out.block_tables = block_tables.data();
    out.tables_cap = block_tables.size();
    out.last_token_indices = last_token_indices.data();
    out.temperatures = temperatures.data();
    out.seeds = seeds.data();
    out.samples_cap = seeds.size();
    if (nvbh_make_batch(nsegs.data(), nsegs.size(), bs, seed, &out))
      return efail("make_batch: %s", nvbh_last_error());
    NvbhBatch batch{};
    batch.token_ids = token_ids.data();
    batch.positions = positions.data();
    batch.sequence_ids = sequence_ids.data();
    batch.slot_mapping = slot_mapping.data();
    batch.rows = out.rows;
    batch.block_tables = block_tables.data();
    batch.block_tables_len = segments.size() * out.table_stride;
    batch.table_stride = out.table_stride;
    batch.last_token_indices = last_token_indices.data();
    batch.temperatures = temperatures.data();
    batch.seeds = seeds.data();
    batch.samples = out.samples;
    size_t decode_rows = 0;
    for (const Segment& seg : segments)
      if (seqs[seg.sequence].is_decode()) decode_rows += seg.end - seg.start;
    const bool all_decode = decode_rows == out.rows;
    batch.is_decode = all_decode ? 1 : 0;

    const auto forward_started = clock::now();
    std::fill(sampled.begin(), sampled.begin() + long(out.samples), std::numeric_limits<uint32_t>::max());
    if (int rc = run(runner, &batch, sampled.data())) return efail("model runner failed (status %d)", rc);
    if (int rc = synchronize()) return rc;
    const double forward_seconds = std::chrono::duration<double>(clock::now() - forward_started).count();
    for (size_t k = 0; k < out.samples; ++k)
      if (sampled[k] > uint32_t(kI32Max)) return efail("model returned a token ID that does not fit in i32");

    if (all_decode) {
      stats.decode_steps += 1;
      stats.decode_tokens += out.rows;
      stats.decode_seconds += forward_seconds;
    } else if (decode_rows == 0) {
      stats.prefill_steps += 1;
      stats.prefill_tokens += out.rows;
      stats.prefill_seconds += forward_seconds;
    } else {
      stats.mixed_steps += 1;
      stats.decode_tokens += decode_rows;
      stats.prefill_tokens += out.rows - decode_rows;
      stats.mixed_seconds += forward_seconds;
    }
    const double now_ms = std::chrono::duration<double, std::milli>(clock::now() - started).count();
    size_t sample_index = 0;
    for (const Segment& seg : segments) {
      Sequence& s = seqs[seg.sequence];
      s.computed = seg.end;
      if (config.prefix_caching) {
        // Publish every page this pass completed (src/runtime.rs:640-648).
        for (size_t logical = seg.start / bs; logical < s.computed / bs; ++logical)
          nvbh_pool_publish(pool, s.blocks[logical], s.tokens.data(), (logical + 1) * bs);
      }
      if (!seg.sample) continue;
      const uint32_t token = sampled[sample_index++];
      s.tokens.push_back(token);
      if (s.first_token_ms < 0) s.first_token_ms = now_ms;
      if (s.previous_token_ms >= 0) s.gaps_ms.push_back(now_ms - s.previous_token_ms);
      s.previous_token_ms = now_ms;
      const bool eos = !s.request->ignore_eos && config.eos_token_id >= 0 && int64_t(token) == config.eos_token_id;
      if (eos || s.generated() == s.request->max_tokens) {
        s.finish_reason = eos ? NVBE_FINISH_EOS : NVBE_FINISH_LENGTH;
        s.latency_ms = now_ms;
        s.status = Status::Finished;
        s.release(pool);
        finished += 1;
      }
    }
    size_t kept = 0;
    for (size_t i : active)
      if (seqs[i].status == Status::Active) active[kept++] = i;
    active.resize(kept);
  }
  return 0;
}

extern "C" {

const char* nvbe_engine_last_error(void) { return g_engine_error; }

int nvbe_engine_create(const NvbeSchedulerConfig* config, NvbeRunFn run, NvbeSyncFn sync, void* runner,
                       NvbeEngine** out) {
  if (int rc = nvbe_scheduler_config_validate(config)) return rc;
  if (!run || !out) return efail("a run function and an output pointer are required");
  NvbeEngine* e = new (std::nothrow) NvbeEngine();
  if (!e) return efail("host allocation failed");
  e->config = *config;
  e->run = run;
  e->sync = sync;
  e->runner = runner;
  e->pool = nvbh_pool_create(config->num_blocks);
  if (!e->pool) {
    delete e;
    return efail("host allocation failed");
  }
  const size_t rows = config->max_batch_tokens, seqs = config->max_sequences;
  const size_t stride = ceil_div(config->max_model_len, config->block_size);
  try {
    for (auto* v : {&e->token_ids, &e->positions, &e->sequence_ids, &e->slot_mapping}) v->resize(rows);
    e->block_tables.resize(seqs * stride);
    e->last_token_indices.resize(seqs);
    e->temperatures.resize(seqs);
    e->seeds.resize(seqs);
    e->sampled.resize(seqs);
  } catch (...) {
    nvbh_pool_destroy(e->pool);
    delete e;
    return efail("host allocation failed");
  }
  *out = e;
  return 0;
}

void nvbe_engine_destroy(NvbeEngine* e) {
  if (!e) return;
  nvbh_pool_destroy(e->pool);
  delete e;
}

int nvbe_engine_generate(NvbeEngine* e, const NvbeRequest* requests, size_t n, uint64_t seed,
                         NvbeRequestOutput* outputs, NvbeRunStats* stats) {
  g_engine_error[0] = 0;
  if (!e || (n && (!requests || !outputs)) || !stats) return efail("invalid generate arguments");
  if (e->failed) return efail("engine is unusable after a model runner failure");
  if (int rc = e->validate_requests(requests, n)) return rc;
  for (size_t i = 0; i < n; ++i)
    if (!outputs[i].token_ids) return efail("output %zu has no token buffer", i);
  if (int rc = e->synchronize()) return rc;
  *stats = NvbeRunStats{};
  const auto started = std::chrono::steady_clock::now();
  std::vector<Sequence> seqs(n);
  for (size_t i = 0; i < n; ++i) {
    seqs[i].request = &requests[i];
    seqs[i].tokens.assign(requests[i].prompt_token_ids, requests[i].prompt_token_ids + requests[i].prompt_len);
  }
  int rc = e->execute(seqs, seed, *stats, started);
  // Cleanup is unconditional, including after a failed forward.
  for (auto& s : seqs) s.release(e->pool);
  if (rc) {
    e->failed = true;
    nvbh_pool_clear_cache(e->pool);
    return rc;
  }
  stats->elapsed_seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - started).count();
  double ttft = 0, latency = 0, gaps = 0;
  size_t ngaps = 0;
  for (size_t i = 0; i < n; ++i) {
    const Sequence& s = seqs[i];
    NvbeRequestOutput& o = outputs[i];
    o.num_tokens = s.generated();
    std::memcpy(o.token_ids, s.tokens.data() + requests[i].prompt_len, o.num_tokens * sizeof(uint32_t));
    o.prompt_tokens = requests[i].prompt_len;
    o.cached_tokens = s.cached_tokens;
    o.ttft_ms = s.first_token_ms < 0 ? 0.0 : s.first_token_ms;
    o.latency_ms = s.latency_ms;
    o.num_gaps = s.gaps_ms.size();
    if (o.inter_token_latencies_ms)
      std::memcpy(o.inter_token_latencies_ms, s.gaps_ms.data(), o.num_gaps * sizeof(double));
    o.finish_reason = s.finish_reason;
    stats->output_tokens += o.num_tokens;
    ttft += o.ttft_ms;
    latency += o.latency_ms;
    for (double g : s.gaps_ms) gaps += g;
    ngaps += s.gaps_ms.size();
  }
  if (stats->elapsed_seconds > 0) stats->output_tokens_per_second = double(stats->output_tokens) / stats->elapsed_seconds;
  if (n) {
    stats->mean_ttft_ms = ttft / double(n);
    stats->mean_latency_ms = latency / double(n);
  }
  if (ngaps) stats->mean_inter_token_latency_ms = gaps / double(ngaps);
  return 0;
}

int nvbe_engine_clear_prefix_cache(NvbeEngine* e) {
  g_engine_error[0] = 0;
  if (!e) return efail("null engine");
  if (nvbh_pool_in_use(e->pool) != 0) return efail("requests still hold KV blocks");
  nvbh_pool_clear_cache(e->pool);
  return 0;
}

size_t nvbe_engine_blocks_in_use(const NvbeEngine* e) { return e ? nvbh_pool_in_use(e->pool) : 0; }

size_t nvbe_engine_cached_keys(const NvbeEngine* e) { return e ? nvbh_pool_cached_keys(e->pool) : 0; }

}  // extern "C"
