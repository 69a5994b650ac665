// CPU oracle for the paged-attention hot path — TEST INFRASTRUCTURE ONLY.
//
// This file restates, in scalar FP32 C++, the reference algorithms that the
// B200 kernels must reproduce. Only tests/, __graft_entry__.smoke() and the
// CPU-baseline leg of bench.py load it, and only as the checker or as the
// timed CPU baseline; the library (libnvb.so) never calls it.
//
// Sources restated (paths relative to the nano-vllm-rs repository):
//  * oracle_attention_native: the CPU FP32 oracle of
//    src/gpu.rs:1430-1466 (gpu_ragged_gqa_matches_cpu), which checks the
//    native kernel nv_attention (kernels/kernels.cu:226-271, 288-354):
//    context = positions[row] + 1, table row = seq_indices[row], score =
//    sum_d q*k / sqrt(dim) accumulated in f32, max-subtracted exp, V summed in
//    token order, divided at the end. Invalid rows give 0 and tokens of
//    invalid pages are skipped, as the native kernel does
//    (kernels/kernels.cu:233-236, 244-248, 264).
//  * oracle_attention_varlen: the FP32 causal oracle of
//    kernels/flash_native/smoke.cu:57-81 over cu_q / kv_lens (query i of a
//    q_len-query group sees kv_len - q_len + i + 1 keys), plus the natural
//    log-sum-exp the FA2 adapter writes to `lse`.
//  * oracle_qkv_rope: qkv_rope_kernel<CACHED> (kernels/kernels.cu:166-211):
//    RMSNorm in f32, BF16 rounding of the normalised value (:185),
//    non-contracted rotate-half products (:203-204), Q to qout, K/V to
//    slots[row] with invalid slots skipped (:189, 206-209).
//  * oracle_rope_cache: rope_cache_kernel (kernels/kernels.cu:213-224).
//  * oracle_bf16_round: round-to-nearest-even f32 -> bf16 as in the test
//    helper of src/gpu.rs:1151-1159.
//
// Known, intended differences from the device reference: the CPU uses the C
// library's sqrtf/expf/powf/sincosf, so results may differ from CUDA's
// approximations by a few ulp; tests therefore compare with tolerances,
// except for the integer slot scatter, which is exact.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

inline float bf(uint16_t h) {
  uint32_t u = uint32_t(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline uint16_t to_bf16(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40);  // quiet NaN
  return uint16_t((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

// One (query row, head) of causal paged attention over `n` keys of table row
// `table`, writing dim floats to out and the natural LSE.
void attend(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int* table, int n, int kvhead,
            int kvh, int dim, int bs, int blocks, float* out, float* lse, std::vector<float>& scores) {
  scores.assign(n, -INFINITY);
  float m = -INFINITY;
  for (int j = 0; j < n; ++j) {
    const int block = table[j / bs];
    if (block < 0 || block >= blocks) continue;
    const size_t base = ((size_t(block) * bs + j % bs) * kvh + kvhead) * dim;
    float dot = 0.0f;
    for (int d = 0; d < dim; ++d) dot += bf(q[d]) * bf(k[base + d]);
    scores[j] = dot / std::sqrt(float(dim));
    m = std::max(m, scores[j]);
  }
  float total = 0.0f;
  for (int j = 0; j < n; ++j) {
    scores[j] = std::isfinite(m) && std::isfinite(scores[j]) ? std::exp(scores[j] - m) : 0.0f;
    total += scores[j];
  }
  for (int d = 0; d < dim; ++d) {
    float val = 0.0f;
    for (int j = 0; j < n; ++j) {
      const int block = table[j / bs];
      if (block < 0 || block >= blocks) continue;
      const size_t base = ((size_t(block) * bs + j % bs) * kvh + kvhead) * dim;
      val += scores[j] * bf(v[base + d]);
    }
    out[d] = total > 0.0f ? val / total : 0.0f;
  }
  if (lse) *lse = total > 0.0f ? m + std::log(total) : -INFINITY;
}

template <class F>
void parallel_for(long long n, int threads, F&& f) {
  if (threads <= 1 || n < 2) {
    for (long long i = 0; i < n; ++i) f(i);
    return;
  }
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([&, t] {
      for (long long i = t; i < n; i += threads) f(i);
    });
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

void oracle_bf16_round(const float* in, uint16_t* out, long long n) {
  for (long long i = 0; i < n; ++i) out[i] = to_bf16(in[i]);
}

// Native-form causal paged GQA (see header comment). out: [rows, qh, dim] f32.
void oracle_attention_native(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int* positions,
                             const int* seqs, const int* tables, float* out, int rows, int qh, int kvh, int dim,
                             int bs, int blocks, int stride, int batch, int max_context, int threads) {
  parallel_for((long long)rows * qh, threads, [&](long long item) {
    std::vector<float> scores;
    const int row = int(item / qh), head = int(item % qh);
    float* o = out + item * dim;
    const int seq = seqs[row];
    const long long ctx = (long long)positions[row] + 1;
    if (seq < 0 || seq >= batch || ctx < 1 || ctx > max_context || ctx > (long long)stride * bs) {
      for (int d = 0; d < dim; ++d) o[d] = 0.0f;
      return;
    }
    attend(q + item * dim, k, v, tables + (size_t)seq * stride, int(ctx), head / (qh / kvh), kvh, dim, bs, blocks,
           o, nullptr, scores);
  });
}

// cu_q / kv_lens form (decode when every group has one query).
// out: [total_q, qh, 128] f32; lse: [(b*qh + h)*max_q + i] natural log.
void oracle_attention_varlen(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int* cu_q,
                             const int* kv_lens, const int* table, float* out, float* lse, int batch, int max_q,
                             int qh, int kvh, int bs, int blocks, int stride, int threads) {
  const int dim = 128;
  const long long total_q = cu_q[batch];
  std::vector<int> seq_of(total_q);
  for (int b = 0; b < batch; ++b)
    for (int r = cu_q[b]; r < cu_q[b + 1]; ++r) seq_of[r] = b;
  parallel_for(total_q * qh, threads, [&](long long item) {
    std::vector<float> scores;
    const int row = int(item / qh), head = int(item % qh);
    const int b = seq_of[row];
    const int qlen = cu_q[b + 1] - cu_q[b], i = row - cu_q[b];
    const long long n = (long long)kv_lens[b] - qlen + i + 1;
    float* o = out + item * dim;
    float* l = lse ? lse + ((long long)b * qh + head) * max_q + i : nullptr;
    if (n < 1 || n > (long long)stride * bs) {
      for (int d = 0; d < dim; ++d) o[d] = 0.0f;
      if (l) *l = -INFINITY;
      return;
    }
    attend(q + item * dim, k, v, table + (size_t)b * stride, int(n), head / (qh / kvh), kvh, dim, bs, blocks, o, l,
           scores);
  });
}

// qkv_rope_kernel<CACHED> restated. qout/kcache/vcache are bf16 buffers
// updated in place (cache entries of invalid slots are left untouched).
void oracle_qkv_rope(const uint16_t* qkv, const uint16_t* qw, const uint16_t* kw, const int* positions,
                     const int* slots, uint16_t* qout, uint16_t* kcache, uint16_t* vcache, int rows, int qh, int kvh,
                     int dim, int bs, int blocks, float eps, float theta, const float* rope_cache,
                     int max_positions, int cached) {
  std::vector<float> normalized(dim);
  const int half = dim / 2;
  for (int row = 0; row < rows; ++row) {
    for (int head = 0; head < qh + kvh; ++head) {
      const bool is_q = head < qh;
      const int local = is_q ? head : head - qh;
      const size_t packed = (size_t)row * (qh + 2 * kvh) * dim;
      const uint16_t* x = qkv + packed + (size_t)head * dim;
      const uint16_t* w = is_q ? qw : kw;
      float sum = 0.0f;
      for (int j = 0; j < dim; ++j) sum += bf(x[j]) * bf(x[j]);
      const float inv_rms = 1.0f / std::sqrt(sum / dim + eps);
      for (int j = 0; j < dim; ++j) normalized[j] = bf(to_bf16(bf(x[j]) * inv_rms * bf(w[j])));
      const int position = positions[row], slot = slots[row];
      const bool valid_slot = slot >= 0 && (long long)slot < (long long)bs * blocks;
      for (int j = 0; j < dim; ++j) {
        const int pair = j % half;
        float c, s;
        if (cached) {
          const bool ok = position >= 0 && position < max_positions;
          c = ok ? rope_cache[(size_t)position * dim + pair] : 1.0f;
          s = ok ? rope_cache[(size_t)position * dim + half + pair] : 0.0f;
        } else {
          const float angle = position * std::pow(theta, -float(2 * pair) / dim);
          s = std::sin(angle);
          c = std::cos(angle);
        }
        // Two separately rounded products, as kernels.cu:203-204.
        volatile float a = normalized[j] * c;
        volatile float b2 = (j < half ? normalized[j + half] : normalized[j - half]) * s;
        const float rotated = j < half ? a - b2 : a + b2;
        if (is_q) {
          qout[((size_t)row * qh + local) * dim + j] = to_bf16(rotated);
        } else if (valid_slot) {
          const size_t base = ((size_t)slot * kvh + local) * dim;
          kcache[base + j] = to_bf16(rotated);
          vcache[base + j] = qkv[packed + (size_t)(qh + kvh + local) * dim + j];
        }
      }
    }
  }
}

void oracle_rope_cache(float* cache, int positions, int dim, float theta) {
  const int half = dim / 2;
  for (int p = 0; p < positions; ++p)
    for (int pair = 0; pair < half; ++pair) {
      const float angle = p * std::pow(theta, -float(2 * pair) / dim);
      cache[(size_t)p * dim + pair] = std::cos(angle);
      cache[(size_t)p * dim + half + pair] = std::sin(angle);
    }
}

int oracle_hardware_threads(void) { return int(std::thread::hardware_concurrency()); }

}  // extern "C"
