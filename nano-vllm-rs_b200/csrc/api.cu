// C ABI of libnvb.so: argument validation, TMA descriptor encoding and
// dispatch. Declarations and the reference entry point each function
// replaces are in include/nvb_attention.h.
//
// Error handling mirrors the reference adapters
// (kernels/flash_native/flash_native.cu:11-58, kernels/kernels.cu:11-25):
// invalid host arguments return -1, a launch error returns the positive
// cudaError_t, and the message goes to a thread-local buffer.
#include <cuda.h>
#include <cuda_runtime.h>

#include <climits>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "internal.cuh"
#include "nvb_attention.h"

namespace nvb {

namespace api_detail {

thread_local char g_last_error[512] = {};

int fail(const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  std::vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
  return -1;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return 0;
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%d)", what, cudaGetErrorString(e), int(e));
  return int(e);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------- TMA maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

struct MapKey {
  const void* base;
  uint64_t dims[3];
  uint64_t strides[2];
  uint32_t box[3];
  int swizzle;
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};

struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    // FNV-1a over the key's bytes (the key is zero-initialised, padding included)
    const unsigned char* b = reinterpret_cast<const unsigned char*>(&k);
    uint64_t h = 1469598103934665603ULL;
    for (size_t i = 0; i < sizeof(MapKey); ++i) h = (h ^ b[i]) * 1099511628211ULL;
    return size_t(h);
  }
};

// Per-thread descriptor cache: a descriptor depends only on the base pointer
// and the geometry, which stay fixed across an engine's steps (a 28-layer
// model uses a few hundred). Descriptors are copied out by value, so a
// later lookup can never change one a caller already holds.
constexpr size_t kMaxCachedMaps = 4096;
thread_local std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

std::mutex g_ctx_mutex;
unsigned long long g_ctx_id[kContextSlots] = {};
unsigned g_ctx_gen[kContextSlots] = {};
unsigned g_ctx_gen_next = 0;
int g_ctx_next = 0;

}  // namespace api_detail

int context_slot(int* slot, unsigned* gen) {
  using namespace api_detail;
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(ptr);
    ptr = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(ptr);
  });
  if (!get_current || !get_id) return int(cudaErrorNotSupported);
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS) return int(cudaErrorDeviceUninitialized);
  if (!ctx) {
    // No context bound to this thread yet: cudaSetDevice binds (and, since
    // CUDA 12, initialises) the current device's primary context.
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);
    if (e != cudaSuccess) return int(e);
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return int(cudaErrorDeviceUninitialized);
  }
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return int(cudaErrorDeviceUninitialized);
  std::lock_guard<std::mutex> lock(g_ctx_mutex);
  for (int i = 0; i < kContextSlots; ++i)
    if (g_ctx_gen[i] && g_ctx_id[i] == id) {
      *slot = i;
      *gen = g_ctx_gen[i];
      return 0;
    }
  // A context not seen before takes the oldest slot.
  const int i = g_ctx_next;
  g_ctx_next = (g_ctx_next + 1) % kContextSlots;
  if (++g_ctx_gen_next == 0) ++g_ctx_gen_next;
  g_ctx_id[i] = id;
  g_ctx_gen[i] = g_ctx_gen_next;
  *slot = i;
  *gen = g_ctx_gen[i];
  return 0;
}

// 3-D BF16 tensor map over [dims[2]][dims[1]][dims[0]] (dims[0] contiguous),
// copied into *out.
int make_map_3d(const void* base, const uint64_t dims[3], const uint64_t strides[2], const uint32_t box[3],
                CUtensorMapSwizzle swizzle, CUtensorMap* out) {
  using namespace api_detail;
  MapKey key{};
  key.base = base;
  std::memcpy(key.dims, dims, sizeof(key.dims));
  std::memcpy(key.strides, strides, sizeof(key.strides));
  std::memcpy(key.box, box, sizeof(key.box));
  key.swizzle = int(swizzle);
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return 0;
  }
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail("cuTensorMapEncodeTiled is unavailable from the CUDA driver");
  CUtensorMap map;
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  const CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                        elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail("cuTensorMapEncodeTiled failed (%d)", int(r));
  if (g_maps.size() >= kMaxCachedMaps) g_maps.clear();
  g_maps.emplace(key, map);
  *out = map;
  return 0;
}

namespace api_detail {

// Decode tiles: [tokens][kv_heads][128] with a {128, 1, kDecodeTile} box.
int kv_decode_map(const void* cache, long long tokens, int kvh, CUtensorMap* out) {
  const uint64_t dims[3] = {128, uint64_t(kvh), uint64_t(tokens)};
  const uint64_t strides[2] = {256, uint64_t(kvh) * 256};
  const uint32_t box[3] = {128, 1, uint32_t(kDecodeTile)};
  return make_map_3d(cache, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE, out);
}

constexpr float kScaleLog2 = 1.4426950408889634f / 11.313708498984761f;  // log2(e) / sqrt(128)

// tcgen05 decode tiles: [tokens][kv_heads][128] with a {64, 1, rows} box
// (rows 128, or 64 for short last tiles), 128B swizzle.
int kv_mma_map(const void* cache, long long tokens, int kvh, CUtensorMap* out, uint32_t rows = 128) {
  const uint64_t dims[3] = {128, uint64_t(kvh), uint64_t(tokens)};
  const uint64_t strides[2] = {256, uint64_t(kvh) * 256};
  const uint32_t box[3] = {64, 1, rows};
  return make_map_3d(cache, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, out);
}

// tcgen05 decode queries: [rows][qh][128] with a {64, 16, 1} box, 128B
// swizzle (one row's 16 heads from the head group's first; heads past qh are
// zero fill).
int q_mma_map(const void* q, int rows, int qh, CUtensorMap* out) {
  const uint64_t dims[3] = {128, uint64_t(qh), uint64_t(rows)};
  const uint64_t strides[2] = {256, uint64_t(qh) * 256};
  const uint32_t box[3] = {64, 16, 1};
  return make_map_3d(q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, out);
}

// `combine` false leaves split-KV partials in lse_accum / out_accum for the
// caller's own combine (the multi-GPU gather path); only the tensor-core
// decode can stop there.
int run_decode(cudaStream_t stream, DecodeParams p, const void* k, const void* v, bool combine = true) {
  const long long tokens = (long long)p.num_blocks * p.block_size;
  CUtensorMap kmap, vmap;
  p.scale_log2 = kScaleLog2;
  if (p.mode == kModeDecode && p.block_size % 128 == 0) {
    if (int rc = kv_mma_map(k, tokens, p.kvh, &kmap)) return rc;
    if (int rc = kv_mma_map(v, tokens, p.kvh, &vmap)) return rc;
    CUtensorMap khalf, vhalf;
    if (int rc = kv_mma_map(k, tokens, p.kvh, &khalf, 64)) return rc;
    if (int rc = kv_mma_map(v, tokens, p.kvh, &vhalf, 64)) return rc;
    p.n_hgroups = (p.qh / p.kvh + 15) / 16;
    // Short contexts (an engine's decode batch: max_k bounded by its model
    // length) take the persistent schedule; long ones one CTA per item,
    // measured faster for them.
    cudaError_t e;
    if (p.max_k > 0 && p.max_k <= kPersistentMaxK) {
      CUtensorMap qmap;
      if (int rc = q_mma_map(p.q, p.rows, p.qh, &qmap)) return rc;
      e = launch_decode_persistent(p, kmap, vmap, khalf, vhalf, qmap, stream);
    } else {
      e = launch_decode_mma(p, kmap, vmap, khalf, vhalf, stream);
    }
    if (e != cudaErrorNotSupported) {
      if (e == cudaSuccess && p.num_splits > 1 && combine) e = launch_combine(p, stream);
      return cuda_status(e, "decode attention launch");
    }
    // NotSupported is returned before any launch: no error state to clear.
  }
  if (!combine) return fail("split partials need the tensor-core decode (block_size a multiple of 128)");
  if (int rc = kv_decode_map(k, tokens, p.kvh, &kmap)) return rc;
  if (int rc = kv_decode_map(v, tokens, p.kvh, &vmap)) return rc;
  p.scale_log2 = kScaleLog2;
  return cuda_status(launch_decode(p, kmap, vmap, stream), "decode attention launch");
}

int paged_fwd_impl(void* stream, const void* q, const void* k, const void* v, void* out, const int* cu_q,
                   const int* kv_lens, const int* block_table, int batch, int total_q, int max_q, int max_k,
                   int q_heads, int kv_heads, int block_size, int table_stride, int num_splits, float* lse,
                   float* lse_accum, float* out_accum, int num_blocks, bool bounded, bool combine = true) {
  g_last_error[0] = 0;
  // Same checks as kernels/flash_native/flash_native.cu:48-58, except the
  // 4096-token context cap, which this implementation does not have.
  if (!q || !k || !v || !out || !cu_q || !kv_lens || !block_table || batch <= 0 || batch > (1 << 20) ||
      total_q < batch || max_q < 1 || max_k < 1 || q_heads <= 0 || q_heads > 256 || kv_heads <= 0 ||
      q_heads % kv_heads || block_size <= 0 || block_size % 256 || table_stride <= 0 ||
      (long long)max_k > (long long)block_size * table_stride ||
      (long long)block_size * table_stride > INT_MAX || (long long)total_q > (long long)batch * max_q ||
      num_splits < 1 || num_splits > 128 || (max_q == 1 && total_q != batch) || (max_q != 1 && num_splits != 1) ||
      (num_splits > 1 && (!lse_accum || !out_accum)))
    return fail("invalid paged attention BF16 hdim128 arguments");
  if (bounded && (num_blocks <= 0 || (long long)num_blocks * block_size > INT_MAX))
    return fail("num_blocks must be positive and num_blocks * block_size must fit in int32");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || (out_accum && !aligned16(out_accum)))
    return fail("q, k, v, out and out_accum must be 16-byte aligned");
  if (!bounded) num_blocks = INT_MAX / block_size;
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  if (max_q > 1) {
    PrefillArgs a{q, k, v, out, cu_q, kv_lens, block_table, lse, batch, total_q, max_q, max_k, q_heads,
                  kv_heads, block_size, table_stride, num_blocks};
    const cudaError_t e = launch_prefill(a, s);
    if (e != cudaErrorNotSupported) return cuda_status(e, "prefill attention launch");
    // Shapes the tcgen05 kernel does not cover run one CTA per query row
    // (launch_prefill returns NotSupported before launching anything).
    DecodeParams p{};
    p.q = static_cast<const __nv_bfloat16*>(q);
    p.out = static_cast<__nv_bfloat16*>(out);
    p.lens = kv_lens;
    p.seq_map = cu_q;
    p.block_table = block_table;
    p.lse = lse;
    p.rows = total_q;
    p.qh = q_heads;
    p.kvh = kv_heads;
    p.block_size = block_size;
    p.table_stride = table_stride;
    p.num_blocks = num_blocks;
    p.batch = batch;
    p.max_context = INT_MAX;
    p.num_splits = 1;
    p.max_q = max_q;
    p.mode = kModeVarlen;
    return run_decode(s, p, k, v);
  }
  DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lens = kv_lens;
  p.seq_map = nullptr;
  p.block_table = block_table;
  p.lse = lse;
  p.lse_accum = lse_accum;
  p.out_accum = out_accum;
  p.rows = batch;
  p.qh = q_heads;
  p.kvh = kv_heads;
  p.block_size = block_size;
  p.table_stride = table_stride;
  p.num_blocks = num_blocks;
  p.batch = batch;
  p.max_context = INT_MAX;
  p.num_splits = num_splits;
  p.max_q = 1;
  p.mode = kModeDecode;
  p.max_k = max_k;
  return run_decode(s, p, k, v, combine);
}

int native_impl(void* stream, const void* q, const void* kc, const void* vc, const int* positions,
                const int* seq_indices, const int* tables, void* out, int rows, int qh, int kvh, int dim, int bs,
                int blocks, int stride, int batch, int max_context, float* scratch, int partitions) {
  g_last_error[0] = 0;
  if (!q || !kc || !vc || !positions || !seq_indices || !tables || !out || rows <= 0 || qh <= 0 || kvh <= 0 ||
      qh % kvh || bs <= 0 || blocks <= 0 || stride <= 0 || batch <= 0 || max_context <= 0)
    return fail("invalid paged attention arguments");
  if (dim != 128) {
    // Other head sizes (kernels/kernels.cu:475-485 dispatch, generic kernel
    // kernels.cu:226-271): the CUDA-core path of generic.cu.
    if (dim < 1 || dim > 512) return fail("head_dim must be in [1, 512] (got %d)", dim);
    if (partitions != 1) return fail("split partitions are supported for head_dim 128 only");
    if ((long long)blocks * bs > INT_MAX) return fail("num_blocks * block_size must fit in int32");
    if ((long long)stride * bs > INT_MAX) return fail("table_stride * block_size must fit in int32");
    return cuda_status(launch_generic_attention(q, kc, vc, out, positions, seq_indices, tables, rows, qh, kvh, dim,
                                                bs, blocks, stride, batch, max_context,
                                                static_cast<cudaStream_t>(stream)),
                       "generic attention launch");
  }
  if (bs % 32) return fail("block_size must be a multiple of 32 (got %d)", bs);
  if ((long long)blocks * bs > INT_MAX) return fail("num_blocks * block_size must fit in int32");
  if (partitions < 1 || partitions > 128 || (partitions > 1 && !scratch))
    return fail("partitions must be in [1, 128] with scratch for more than one");
  if (!aligned16(q) || !aligned16(kc) || !aligned16(vc) || !aligned16(out) || (scratch && !aligned16(scratch)))
    return fail("q, caches, out and scratch must be 16-byte aligned");
  DecodeParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lens = positions;
  p.seq_map = seq_indices;
  p.block_table = tables;
  p.lse = nullptr;
  // Scratch layout (opaque to callers): FP32 partials [P][rows][qh][128]
  // followed by their LSEs [P][rows][qh]; fits rows*qh*P*(128+2) floats.
  p.out_accum = partitions > 1 ? scratch : nullptr;
  p.lse_accum = partitions > 1 ? scratch + (size_t)partitions * rows * qh * 128 : nullptr;
  p.rows = rows;
  p.qh = qh;
  p.kvh = kvh;
  p.block_size = bs;
  p.table_stride = stride;
  p.num_blocks = blocks;
  p.batch = batch;
  p.max_context = max_context;
  p.num_splits = partitions;
  p.max_q = 1;
  p.mode = kModeNative;
  return run_decode(static_cast<cudaStream_t>(stream), p, kc, vc);
}

}  // namespace api_detail
}  // namespace nvb

using namespace nvb;
using namespace nvb::api_detail;

extern "C" {

const char* nvb_last_error(void) { return g_last_error; }

const char* nvb_version(void) { return "nvb 0.1 sm_100a"; }

int nvb_paged_fwd(void* stream, const void* q, const void* k, const void* v, void* out, const int* cu_q,
                  const int* kv_lens, const int* block_table, int batch, int total_q, int max_q, int max_k,
                  int q_heads, int kv_heads, int block_size, int table_stride, int num_splits, float* lse,
                  float* lse_accum, float* out_accum) {
  if (!lse) return fail("invalid paged attention BF16 hdim128 arguments");
  return paged_fwd_impl(stream, q, k, v, out, cu_q, kv_lens, block_table, batch, total_q, max_q, max_k, q_heads,
                        kv_heads, block_size, table_stride, num_splits, lse, lse_accum, out_accum, 0, false);
}

int nvb_paged_fwd_ex(void* stream, const void* q, const void* k, const void* v, void* out, const int* cu_q,
                     const int* kv_lens, const int* block_table, int batch, int total_q, int max_q, int max_k,
                     int q_heads, int kv_heads, int block_size, int table_stride, int num_splits, float* lse,
                     float* lse_accum, float* out_accum, int num_blocks) {
  return paged_fwd_impl(stream, q, k, v, out, cu_q, kv_lens, block_table, batch, total_q, max_q, max_k, q_heads,
                        kv_heads, block_size, table_stride, num_splits, lse, lse_accum, out_accum, num_blocks, true);
}

int nvb_num_splits(int batch, int q_heads, int kv_heads, int max_k, int num_sms) {
  if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || max_k <= 0 || num_sms <= 0 ||
      num_sms > 1024)
    return 0;
  int group = q_heads / kv_heads, gc = 1;
  for (int c = 8; c >= 1; --c)
    if (group % c == 0) { gc = c; break; }
  // CTAs per (sequence, kv head): 16-head groups in the tensor-core decode
  // past 16 heads, the CUDA-core decode's head chunks below.
  const long long units = group > 16 ? (group + 15) / 16 : group / gc;
  const long long work = (long long)batch * kv_heads * units;
  const long long target = 2LL * num_sms;  // two resident CTAs per SM
  if (work >= target) return 1;
  // The most splits that still fit one wave of resident CTAs: a split count
  // one past it leaves a sparse second wave too small to keep HBM busy
  // (4 x 8 heads x 10 splits = 320 CTAs on 296 slots ran at 0.62 of copy
  // bandwidth).
  long long splits = target / work;
  const long long max_by_len = (max_k + 255) / 256;  // keep >= 256 keys per split
  if (splits > max_by_len) splits = max_by_len;
  if (splits > 128) splits = 128;
  return splits < 1 ? 1 : int(splits);
}

int nvb_attention(void* stream, const void* q, const void* kcache, const void* vcache, const int* positions,
                  const int* seq_indices, const int* tables, void* out, int rows, int q_heads, int kv_heads,
                  int head_dim, int block_size, int num_blocks, int table_stride, int batch, int max_context) {
  return native_impl(stream, q, kcache, vcache, positions, seq_indices, tables, out, rows, q_heads, kv_heads,
                     head_dim, block_size, num_blocks, table_stride, batch, max_context, nullptr, 1);
}

int nvb_attention_splitkv(void* stream, const void* q, const void* kcache, const void* vcache,
                          const int* positions, const int* seq_indices, const int* tables, void* out, int rows,
                          int q_heads, int kv_heads, int head_dim, int block_size, int num_blocks,
                          int table_stride, int batch, int max_context, float* scratch, int partitions) {
  return native_impl(stream, q, kcache, vcache, positions, seq_indices, tables, out, rows, q_heads, kv_heads,
                     head_dim, block_size, num_blocks, table_stride, batch, max_context, scratch, partitions);
}

static int qkv_rope_common(void* stream, bool cached, const void* qkv, const void* qw, const void* kw,
                           const int* positions, const int* slots, void* qout, void* kc, void* vc, int rows, int qh,
                           int kvh, int dim, int bs, int blocks, float eps, float theta, const float* rope_cache,
                           int max_positions) {
  g_last_error[0] = 0;
  if (!qkv || !qw || !kw || !positions || !slots || !qout || !kc || !vc || rows <= 0 || qh <= 0 || kvh <= 0 ||
      bs <= 0 || blocks <= 0 || !(eps > 0.0f) || !std::isfinite(eps))
    return fail("invalid fused qkv rope arguments");
  if (dim != 128) return fail("only head_dim 128 is supported (got %d)", dim);
  if ((long long)bs * blocks > INT_MAX) return fail("KV slot count exceeds int32");
  if (cached && (!rope_cache || max_positions <= 0)) return fail("rope cache and max_positions are required");
  if (!cached && (!(theta > 0.0f) || !std::isfinite(theta))) return fail("theta must be positive and finite");
  return cuda_status(launch_qkv_rope(static_cast<cudaStream_t>(stream), cached, qkv, qw, kw, positions, slots, qout,
                                     kc, vc, rows, qh, kvh, bs, blocks, eps, theta, rope_cache, max_positions),
                     "fused qkv rope launch");
}

int nvb_qkv_rope_cached(void* stream, const void* qkv, const void* q_weight, const void* k_weight,
                        const int* positions, const int* slots, void* qout, void* kcache, void* vcache, int rows,
                        int q_heads, int kv_heads, int head_dim, int block_size, int num_blocks, float eps,
                        const float* rope_cache, int max_positions) {
  return qkv_rope_common(stream, true, qkv, q_weight, k_weight, positions, slots, qout, kcache, vcache, rows,
                         q_heads, kv_heads, head_dim, block_size, num_blocks, eps, 1.0f, rope_cache, max_positions);
}

int nvb_qkv_rope(void* stream, const void* qkv, const void* q_weight, const void* k_weight, const int* positions,
                 const int* slots, void* qout, void* kcache, void* vcache, int rows, int q_heads, int kv_heads,
                 int head_dim, int block_size, int num_blocks, float eps, float theta) {
  return qkv_rope_common(stream, false, qkv, q_weight, k_weight, positions, slots, qout, kcache, vcache, rows,
                         q_heads, kv_heads, head_dim, block_size, num_blocks, eps, theta, nullptr, 0);
}

int nvb_rope_cache(void* stream, float* cache, int positions, int head_dim, float theta) {
  g_last_error[0] = 0;
  if (!cache || positions <= 0 || head_dim <= 0 || head_dim % 2 || !(theta > 0.0f) || !std::isfinite(theta))
    return fail("invalid rope cache arguments");
  return cuda_status(launch_rope_cache(static_cast<cudaStream_t>(stream), cache, positions, head_dim, theta),
                     "rope cache launch");
}

int nvb_capture_begin(void* stream) {
  return cuda_status(cudaStreamBeginCapture(static_cast<cudaStream_t>(stream), cudaStreamCaptureModeThreadLocal),
                     "cudaStreamBeginCapture");
}

int nvb_capture_end(void* stream, void** graph) {
  if (!graph) return fail("graph output pointer is null");
  cudaGraph_t g = nullptr;
  int rc = cuda_status(cudaStreamEndCapture(static_cast<cudaStream_t>(stream), &g), "cudaStreamEndCapture");
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  cudaGraphExec_t exec = nullptr;
  rc = cuda_status(cudaGraphInstantiate(&exec, g, 0), "cudaGraphInstantiate");
  cudaGraphDestroy(g);
  *graph = rc ? nullptr : static_cast<void*>(exec);
  return rc;
}

void nvb_capture_abort(void* stream) {
  cudaGraph_t g = nullptr;
  cudaStreamEndCapture(static_cast<cudaStream_t>(stream), &g);
  if (g) cudaGraphDestroy(g);
}

int nvb_graph_replay(void* graph, void* stream) {
  if (!graph) return fail("graph is null");
  return cuda_status(cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph), static_cast<cudaStream_t>(stream)),
                     "cudaGraphLaunch");
}

void nvb_graph_destroy(void* graph) {
  if (graph) cudaGraphExecDestroy(static_cast<cudaGraphExec_t>(graph));
}

int nvb_device_error(int* code) {
  if (!code) return fail("code pointer is null");
  return cuda_status(cudaMemcpyFromSymbol(code, g_nvb_device_error, sizeof(int)), "read device error word");
}

int nvb_clear_device_error(void) {
  const int zero = 0;
  return cuda_status(cudaMemcpyToSymbol(g_nvb_device_error, &zero, sizeof(int)), "clear device error word");
}

}  // extern "C"
