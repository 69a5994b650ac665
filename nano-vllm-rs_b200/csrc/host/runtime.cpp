// Host-side metadata of the paged attention path (see include/nvb_host.h).
//
// Restates, in C++, the integer logic of the reference's Rust host that
// produces what the kernels consume:
//   flash_metadata          src/model.rs:234-267
//   MetadataLayout new/pack src/model.rs:271-358
//   validate_batch          src/model.rs:820-921
//   BlockPool               src/runtime.rs:192-296
//   make_batch              src/runtime.rs:728-777
//   sampling_seed           src/runtime.rs:782-790
// Integer outputs are bit-exact with the reference. The prefix hash is this
// library's own (FNV-1a); the reference's SipHash value never leaves the pool
// because lookups compare the full token key.
#include "nvb_host.h"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <limits>
#include <new>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace {

thread_local char g_error[512] = {};

int fail(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  std::vsnprintf(g_error, sizeof(g_error), fmt, args);
  va_end(args);
  return -1;
}

constexpr long long kI32Max = std::numeric_limits<int32_t>::max();

uint64_t mix64(uint64_t v) {  // SplitMix64 finaliser (Steele, Lea, Flood 2014)
  v += 0x9e3779b97f4a7c15ULL;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ULL;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebULL;
  return v ^ (v >> 31);
}

uint64_t prefix_hash(const uint32_t* tokens, size_t n) {
  uint64_t h = 1469598103934665603ULL ^ uint64_t(n);
  for (size_t i = 0; i < n; ++i) {
    h ^= tokens[i];
    h *= 1099511628211ULL;
  }
  return h;
}

template <class T>
void put(uint8_t* staging, size_t offset, T value) {
  std::memcpy(staging + offset, &value, sizeof(T));
}

}  // namespace

struct NvbhBlockPool {
  struct Block {
    size_t references = 0;
    bool has_prefix = false;
    uint64_t hash = 0;
    std::vector<uint32_t> tokens;
    uint64_t last_used = 0;
  };
  std::vector<Block> blocks;
  std::unordered_map<uint64_t, std::vector<int>> by_hash;
  uint64_t clock = 0;
  size_t free_count = 0;  // pages with no references, kept so available() is O(1)

  void touch(int b) {
    if (clock != std::numeric_limits<uint64_t>::max()) ++clock;  // saturating, as the reference
    blocks[b].last_used = clock;
  }
  void invalidate(int b) {
    Block& blk = blocks[b];
    if (!blk.has_prefix) return;
    auto it = by_hash.find(blk.hash);
    if (it != by_hash.end()) {
      auto& v = it->second;
      for (size_t i = 0; i < v.size();) {
        if (v[i] == b) v.erase(v.begin() + long(i)); else ++i;
      }
      if (v.empty()) by_hash.erase(it);
    }
    blk.has_prefix = false;
    blk.tokens.clear();
  }
  int find(const uint32_t* t, size_t n) const {
    auto it = by_hash.find(prefix_hash(t, n));
    if (it == by_hash.end()) return -1;
    for (int id : it->second) {
      const Block& blk = blocks[id];
      if (blk.has_prefix && blk.tokens.size() == n && (n == 0 || std::memcmp(blk.tokens.data(), t, n * 4) == 0))
        return id;
    }
    return -1;
  }
};

extern "C" {

const char* nvbh_last_error(void) { return g_error; }

int nvbh_flash_metadata(const int32_t* positions, const int32_t* sequence_ids, size_t rows, size_t sequences,
                        int32_t* cu_q, int32_t* kv_lens, size_t* max_q) {
  g_error[0] = 0;
  if ((rows && (!positions || !sequence_ids)) || !cu_q || !kv_lens || !max_q) return fail("null metadata pointer");
  size_t row = 0, mq = 0;
  cu_q[0] = 0;
  for (size_t seq = 0; seq < sequences; ++seq) {
    const size_t start = row;
    while (row < rows && sequence_ids[row] == (long long)seq) {
      if (row > start && (long long)positions[row] != (long long)positions[row - 1] + 1)
        return fail("FlashAttention queries must have consecutive positions");
      ++row;
    }
    if (row == start) return fail("FlashAttention requires nonempty query groups in sequence order");
    if (row - start > mq) mq = row - start;
    if ((long long)row > kI32Max) return fail("query offset exceeds i32");
    cu_q[seq + 1] = int32_t(row);
    const long long len = (long long)positions[row - 1] + 1;
    if (len > kI32Max) return fail("KV length overflow");
    kv_lens[seq] = int32_t(len);
  }
  if (row != rows) return fail("FlashAttention query groups are out of order");
  *max_q = mq;
  return 0;
}

int nvbh_metadata_layout(size_t tokens, size_t sequences, size_t table_stride, NvbhMetadataLayout* out) {
  g_error[0] = 0;
  if (!out) return fail("null layout pointer");
  size_t cursor = 0;
  const size_t counts[NVBH_META_FIELDS] = {tokens, tokens, tokens, tokens, 0, sequences, sequences, sequences,
                                           sequences + 1, sequences};
  const size_t widths[NVBH_META_FIELDS] = {4, 4, 4, 4, 4, 4, 4, 8, 4, 4};
  if (table_stride && sequences > std::numeric_limits<size_t>::max() / table_stride)
    return fail("block table size overflow");
  for (int f = 0; f < NVBH_META_FIELDS; ++f) {
    const size_t count = f == NVBH_META_TABLES ? sequences * table_stride : counts[f];
    if (cursor > std::numeric_limits<size_t>::max() - 7) return fail("metadata alignment overflow");
    const size_t start = (cursor + 7) & ~size_t(7);
    if (count > (std::numeric_limits<size_t>::max() - start) / widths[f]) return fail("metadata extent overflow");
    out->start[f] = start;
    cursor = start + count * widths[f];
    out->end[f] = cursor;
  }
  out->bytes = cursor;
  return 0;
}

int nvbh_metadata_pack(const NvbhMetadataLayout* layout, uint8_t* staging, size_t staging_bytes,
                       const NvbhBatch* batch, size_t sequences, size_t table_stride, const int32_t* cu_q,
                       const int32_t* kv_lens) {
  g_error[0] = 0;
  if (!layout || !staging || !batch) return fail("null pack argument");
  if (staging_bytes < layout->bytes) return fail("staging buffer smaller than the layout");
  const size_t rows = batch->rows;
  if (rows * 4 > layout->end[NVBH_META_TOKENS] - layout->start[NVBH_META_TOKENS])
    return fail("batch has more tokens than the layout");
  if (sequences * table_stride * 4 > layout->end[NVBH_META_TABLES] - layout->start[NVBH_META_TABLES])
    return fail("block tables exceed the layout");
  if (batch->table_stride > table_stride || batch->block_tables_len < sequences * batch->table_stride)
    return fail("invalid block table shape");
  if (batch->samples * 4 > layout->end[NVBH_META_LAST_INDICES] - layout->start[NVBH_META_LAST_INDICES])
    return fail("batch has more samples than the layout");
  for (size_t i = 0; i < rows; ++i) {
    put(staging, layout->start[NVBH_META_TOKENS] + 4 * i, batch->token_ids[i]);
    put(staging, layout->start[NVBH_META_POSITIONS] + 4 * i, batch->positions[i]);
    put(staging, layout->start[NVBH_META_SEQUENCES] + 4 * i, batch->sequence_ids[i]);
    put(staging, layout->start[NVBH_META_SLOTS] + 4 * i, batch->slot_mapping[i]);
  }
  std::memset(staging + layout->start[NVBH_META_TABLES], 0xff, sequences * table_stride * 4);
  for (size_t s = 0; s < sequences; ++s)
    for (size_t c = 0; c < batch->table_stride; ++c)
      put(staging, layout->start[NVBH_META_TABLES] + (s * table_stride + c) * 4,
          batch->block_tables[s * batch->table_stride + c]);
  for (size_t i = 0; i < batch->samples; ++i) {
    put(staging, layout->start[NVBH_META_LAST_INDICES] + 4 * i, batch->last_token_indices[i]);
    put(staging, layout->start[NVBH_META_TEMPERATURES] + 4 * i, batch->temperatures[i]);
    put(staging, layout->start[NVBH_META_SEEDS] + 8 * i, batch->seeds[i]);
  }
  if (cu_q)
    for (size_t i = 0; i <= sequences; ++i) put(staging, layout->start[NVBH_META_CU_Q] + 4 * i, cu_q[i]);
  if (kv_lens)
    for (size_t i = 0; i < sequences; ++i) put(staging, layout->start[NVBH_META_KV_LENS] + 4 * i, kv_lens[i]);
  return 0;
}

int nvbh_validate_batch(const NvbhBatch* b, const NvbhLimits* lim, size_t* rows_out, size_t* sequences_out,
                        size_t* samples_out) {
  g_error[0] = 0;
  if (!b || !lim) return fail("null batch or limits");
  const size_t rows = b->rows, samples = b->samples;
  if (rows == 0 || rows > lim->max_batch_tokens) return fail("batch token count is outside model capacity");
  if (!b->token_ids || !b->positions || !b->sequence_ids || !b->slot_mapping) return fail("token metadata lengths differ");
  if (!(b->table_stride > 0 && b->table_stride <= lim->table_stride && b->block_tables_len % b->table_stride == 0))
    return fail("invalid block table shape");
  const size_t sequences = b->block_tables_len / b->table_stride;
  if (!(sequences > 0 && sequences <= lim->max_sequences)) return fail("batch sequence count exceeds capacity");
  if (samples > sequences) return fail("invalid sampling metadata lengths");
  for (size_t i = 0; i < rows; ++i)
    if (b->token_ids[i] < 0 || size_t(b->token_ids[i]) >= lim->vocab_size)
      return fail("token id outside model vocabulary");
  for (size_t i = 0; i < samples; ++i)
    if (b->last_token_indices[i] < 0 || size_t(b->last_token_indices[i]) >= rows) return fail("sample row outside batch");
  for (size_t i = 0; i < samples; ++i)
    if (!std::isfinite(b->temperatures[i]) || b->temperatures[i] < 0.0f)
      return fail("temperature must be finite and nonnegative");
  std::unordered_set<size_t> seen;
  seen.reserve(rows * 2);
  std::vector<long long> max_pos(sequences, -1);
  for (size_t row = 0; row < rows; ++row) {
    const long long position = b->positions[row], sequence = b->sequence_ids[row];
    if (position < 0 || size_t(position) >= lim->max_model_len) return fail("token position exceeds max_model_len");
    if (sequence < 0 || size_t(sequence) >= sequences) return fail("token sequence index outside block tables");
    const size_t column = size_t(position) / lim->block_size;
    if (column >= b->table_stride) return fail("block table does not cover token position");
    const long long block = b->block_tables[size_t(sequence) * b->table_stride + column];
    if (block < 0 || size_t(block) >= lim->num_blocks) return fail("invalid physical KV block");
    const size_t expected = size_t(block) * lim->block_size + size_t(position) % lim->block_size;
    if (b->slot_mapping[row] < 0 || size_t(b->slot_mapping[row]) != expected)
      return fail("KV slot mapping disagrees with block table");
    if (!seen.insert(expected).second) return fail("two input tokens write the same KV slot");
    if (position > max_pos[size_t(sequence)]) max_pos[size_t(sequence)] = position;
  }
  for (size_t s = 0; s < sequences; ++s) {
    if (max_pos[s] < 0) continue;
    for (size_t c = 0; c <= size_t(max_pos[s]) / lim->block_size; ++c) {
      const long long block = b->block_tables[s * b->table_stride + c];
      if (block < 0 || size_t(block) >= lim->num_blocks) return fail("missing KV block in causal context");
    }
  }
  if (rows_out) *rows_out = rows;
  if (sequences_out) *sequences_out = sequences;
  if (samples_out) *samples_out = samples;
  return 0;
}

NvbhBlockPool* nvbh_pool_create(size_t num_blocks) {
  NvbhBlockPool* p = new (std::nothrow) NvbhBlockPool();
  if (p) {
    p->blocks.resize(num_blocks);
    p->free_count = num_blocks;
  }
  return p;
}

void nvbh_pool_destroy(NvbhBlockPool* pool) { delete pool; }

int nvbh_pool_allocate(NvbhBlockPool* p) {
  int best = -1;
  for (size_t i = 0; i < p->blocks.size(); ++i) {
    const auto& b = p->blocks[i];
    if (b.references != 0) continue;
    if (best < 0) { best = int(i); continue; }
    const auto& c = p->blocks[size_t(best)];
    // empty pages first, then least recently used; ties keep the lowest id
    if (b.has_prefix < c.has_prefix || (b.has_prefix == c.has_prefix && b.last_used < c.last_used)) best = int(i);
  }
  if (best < 0) return -1;
  p->invalidate(best);
  p->blocks[size_t(best)].references = 1;
  p->free_count -= 1;
  p->touch(best);
  return best;
}

void nvbh_pool_release(NvbhBlockPool* p, int block) {
  if (block < 0 || size_t(block) >= p->blocks.size() || p->blocks[size_t(block)].references == 0) return;
  p->blocks[size_t(block)].references -= 1;
  if (p->blocks[size_t(block)].references == 0) p->free_count += 1;
  p->touch(block);
}

int nvbh_pool_find(const NvbhBlockPool* p, const uint32_t* tokens, size_t n) { return p->find(tokens, n); }

int nvbh_pool_find_and_retain(NvbhBlockPool* p, const uint32_t* tokens, size_t n) {
  const int b = p->find(tokens, n);
  if (b < 0) return -1;
  if (p->blocks[size_t(b)].references == 0) p->free_count -= 1;
  p->blocks[size_t(b)].references += 1;
  p->touch(b);
  return b;
}

void nvbh_pool_publish(NvbhBlockPool* p, int block, const uint32_t* prefix, size_t n) {
  if (block < 0 || size_t(block) >= p->blocks.size()) return;
  auto& b = p->blocks[size_t(block)];
  if (b.has_prefix) return;  // already keyed by the same prefix
  b.has_prefix = true;
  b.hash = prefix_hash(prefix, n);
  b.tokens.assign(prefix, prefix + n);
  p->by_hash[b.hash].push_back(block);
  p->touch(block);
}

size_t nvbh_pool_available(const NvbhBlockPool* p) { return p->free_count; }

size_t nvbh_pool_in_use(const NvbhBlockPool* p) { return p->blocks.size() - nvbh_pool_available(p); }

size_t nvbh_pool_references(const NvbhBlockPool* p, int block) {
  return (block < 0 || size_t(block) >= p->blocks.size()) ? 0 : p->blocks[size_t(block)].references;
}

size_t nvbh_pool_cached_keys(const NvbhBlockPool* p) { return p->by_hash.size(); }

void nvbh_pool_clear_cache(NvbhBlockPool* p) {
  p->by_hash.clear();
  for (auto& b : p->blocks) {
    b.has_prefix = false;
    b.tokens.clear();
  }
}

void nvbh_pool_force_hash_entry(NvbhBlockPool* p, const uint32_t* prefix, size_t n, int block) {
  p->by_hash[prefix_hash(prefix, n)].push_back(block);
}

int nvbh_make_batch(const NvbhSegment* segs, size_t n, size_t block_size, uint64_t seed, NvbhBatchOut* out) {
  g_error[0] = 0;
  if (!out || (n && !segs) || block_size == 0) return fail("invalid make_batch arguments");
  size_t stride = 0, rows = 0, samples = 0;
  for (size_t i = 0; i < n; ++i) {
    const NvbhSegment& s = segs[i];
    if (s.num_blocks > stride) stride = s.num_blocks;
    if (s.end < s.start || s.end > s.num_tokens) return fail("segment range outside the sequence");
    if (s.end > 0 && (s.end - 1) / block_size >= s.num_blocks) return fail("segment positions outside its pages");
    rows += s.end - s.start;
    samples += s.sample ? 1 : 0;
  }
  if (rows > out->rows_cap || n * stride > out->tables_cap || samples > out->samples_cap)
    return fail("make_batch output capacity too small (rows %zu, tables %zu, samples %zu)", rows, n * stride, samples);
  if (rows > size_t(kI32Max)) return fail("batch dimensions must fit in i32");
  size_t r = 0, t = 0, k = 0;
  for (size_t i = 0; i < n; ++i) {
    const NvbhSegment& s = segs[i];
    for (size_t pos = s.start; pos < s.end; ++pos) {
      const long long physical = s.blocks[pos / block_size];
      const long long slot = physical * (long long)block_size + (long long)(pos % block_size);
      if (physical < 0 || slot > kI32Max) return fail("KV slot indices must fit in i32");
      out->token_ids[r] = int32_t(s.tokens[pos]);
      out->positions[r] = int32_t(pos);
      out->sequence_ids[r] = int32_t(i);
      out->slot_mapping[r] = int32_t(slot);
      ++r;
    }
    for (size_t c = 0; c < stride; ++c) out->block_tables[t++] = c < s.num_blocks ? s.blocks[c] : -1;
    if (s.sample) {
      out->last_token_indices[k] = int32_t(r) - 1;
      out->temperatures[k] = s.temperature;
      out->seeds[k] = nvbh_sampling_seed(seed, s.request_id, s.generated);
      ++k;
    }
  }
  out->rows = r;
  out->table_stride = stride;
  out->samples = k;
  return 0;
}

uint64_t nvbh_sampling_seed(uint64_t base, uint64_t request_id, uint64_t generated) {
  return mix64(mix64(base) ^ mix64(request_id) ^ mix64(generated));
}

}  // extern "C"
