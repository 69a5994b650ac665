// Multi-GPU decode over kv-head shards: the split-KV combine fused with the
// all-gather of the outputs.
//
// Long contexts (4 x 32768 tokens, 64q/8kv) are sharded over the GPUs of a
// node by kv head: rank r owns kv heads [r * kvh_local, (r + 1) * kvh_local)
// and the query heads of their groups, so its decode reads only its share of
// the KV cache. Every rank then needs the whole [batch, q_heads, 128] output.
// Instead of a separate collective after the decode, the combine kernel below
// stores each (sequence, head) result straight into every rank's output
// buffer (peer stores over NVLink through CUDA IPC mappings), and a per-step
// epoch flag is exchanged with every peer (by a one-warp barrier kernel in
// the host-epoch form, by the combine's last CTA in the capturable form), so
// that when a rank's stream moves on, all peers' stores into its buffer have
// landed.
//
// The reference is single-GPU (its README: no NCCL, MPI or tensor
// parallelism); this path has no counterpart there. No TMA, no multicast and
// no library kernel touches peer memory: only plain stores and the flags.
// The barrier's waits are bounded (kWaitCycles) and record kErrGatherWait.
#include "internal.cuh"
#include "combine.cuh"

namespace nvb {

namespace gather_detail {

constexpr int kMaxRanks = 8;

struct PeerPtrs {
  __nv_bfloat16* out[2][kMaxRanks];  // two output sets, each rank's [rows, qh_total, 128]
  unsigned int* flag[kMaxRanks];     // each rank's flags: slot p = last epoch rank p signalled there
};

// Epoch of the step being run: the host's, or (counter != null) one past the
// rank's device counter, which the barrier kernel advances at the end of the
// step. The step's results go to output set `epoch & 1` in the counter form.
__device__ __forceinline__ unsigned int step_epoch(unsigned int host_epoch, const unsigned int* counter) {
  return counter ? *counter + 1u : host_epoch;
}

// Lanes p < world: signal `epoch` into rank p's slot `rank`, then wait (bounded)
// until rank p's epoch has arrived in this rank's slot p. kFence: a full
// system-scope fence before the releasing store (the host-epoch barrier
// kernel, whose ordering with the combine grid comes from griddepcontrol.wait);
// without it the store's own release semantics order what precedes it.
template <bool kFence>
__device__ __forceinline__ void exchange_epoch(const PeerPtrs& peers, int world, int rank, unsigned int epoch,
                                               int lane) {
  if (lane >= world) return;
  if constexpr (kFence) __threadfence_system();
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peers.flag[lane] + rank), "r"(epoch) : "memory");
  const unsigned int* mine = peers.flag[rank] + lane;
  const long long start = clock64();
  for (;;) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
    if (int(v - epoch) >= 0) break;  // epochs only grow (wrap-safe)
    if (clock64() - start > kWaitCycles) {
      record_error(kErrGatherWait);
      break;
    }
    __nanosleep(100);
  }
}

// W warps per (row, local head) item (combine.cuh). splits > 1: weights
// split s by exp(lse_s - max lse) exactly as combine_kernel (decode.cu) does;
// splits == 1: copies the local decode output. The result goes to every rank
// at head offset head_offset (= rank * qh local).
// kBarrier (the counter form): the CTA that finishes last (a done count in
// the rank's flag slot world + 1) runs the epoch exchange itself, advances
// the device epoch and resets the count, so the step needs no separate
// barrier launch.
//
// Ordering of the counter form, in the PTX memory model (causality order is
// transitive; each synchronising pair needs only a scope that holds both
// threads): a CTA's peer stores precede its thread 0's count by bar.sync; the
// count is an acquire-release RMW at GPU scope, and every CTA that counts runs
// on this GPU, so each count synchronises with the last CTA's; that CTA's
// bar.sync then orders them before each lane's st.release.sys of the epoch
// flag, which is cumulative, and a peer that acquires the flag at system scope
// sees every store of the grid. A system-scope fence in each CTA instead
// measured ~4 us per step (it waits for the CTA's NVLink stores to complete),
// the GPU-scope count ~0.9 us.
template <bool kBarrier, int W>
__global__ void __launch_bounds__(combine_detail::kCombineThreads)
    combine_gather_kernel(const float* __restrict__ lse_accum, const float* __restrict__ out_accum,
                          const __nv_bfloat16* __restrict__ local_out, int rows, int qh, int splits, PeerPtrs peers,
                          int world, int head_offset, int qh_total, unsigned int* counter, int rank) {
  // Launched as a programmatic dependent of the decode grid (see
  // nvb_paged_decode_gather): the barrier kernel after it may be scheduled
  // now, and this grid waits for the decode to complete before reading.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The step's epoch (counter form), loaded once: its latency hides under the
  // combine's loads, and the last CTA reuses it for the exchange.
  const unsigned int epoch = counter ? step_epoch(0, counter) : 0u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = warp % W;
  const long long item = (long long)blockIdx.x * (combine_detail::kCombineThreads / 32 / W) + warp / W;
  const bool live = item < (long long)rows * qh;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float total = 0.0f, mx = -INFINITY;
  if (live && splits > 1)
    combine_detail::combine_share<W>(lse_accum, out_accum, item, (long long)rows * qh, splits, sub, lane, acc, total,
                                     mx);
  combine_detail::combine_gather_shares<W>(acc, total, warp, lane, sub);
  if (live && sub == 0) {
    uint2 packed;
    if (splits > 1) {
      const float inv = total > 0.0f ? 1.0f / total : 0.0f;
      packed.x = pack_bf16x2(acc.x * inv, acc.y * inv);
      packed.y = pack_bf16x2(acc.z * inv, acc.w * inv);
    } else {
      packed = *reinterpret_cast<const uint2*>(local_out + item * 128 + lane * 4);
    }
    const long long row = item / qh, h = item - row * qh;
    const long long dst = (row * qh_total + head_offset + h) * 128 + lane * 4;
    const int set = int(epoch & 1u);
    for (int p = 0; p < world; ++p) *reinterpret_cast<uint2*>(peers.out[set][p] + dst) = packed;
  }
  if constexpr (!kBarrier) __threadfence_system();  // the stores are visible to the peers before this thread ends
  if constexpr (kBarrier) {
    __shared__ int last;
    __syncthreads();
    unsigned int* done = counter + 1;
    if (threadIdx.x == 0) {
      unsigned int prev;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(done) : "memory");
      last = prev == unsigned(gridDim.x) - 1u;
    }
    __syncthreads();
    if (!last || threadIdx.x >= 32) return;
    exchange_epoch<false>(peers, world, rank, epoch, lane);
    __syncwarp();
    if (lane == 0) {
      *done = 0u;
      *counter = epoch;
    }
  }
}

// One warp: lane p writes this rank's epoch into rank p's flag slot `rank`,
// then waits until rank p's epoch has arrived in this rank's slot p. In the
// counter form lane 0 then advances the device counter to this epoch.
__global__ void gather_barrier_kernel(PeerPtrs peers, int world, int rank, unsigned int host_epoch,
                                      unsigned int* counter) {
  // Every store of the combine grid before it is complete and visible before
  // this rank signals its peers (programmatic dependent launch).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x;
  const unsigned int epoch = step_epoch(host_epoch, counter);
  exchange_epoch<true>(peers, world, rank, epoch, lane);
  __syncwarp();
  if (counter && lane == 0) *counter = epoch;
}

}  // namespace gather_detail

}  // namespace nvb

// ------------------------------------------------------------ C ABI
// Peer buffers: one cudaMalloc'd region per rank, shared with the other ranks
// of the node through CUDA IPC (no multicast object is created).

extern "C" int nvb_peer_buffer_create(size_t bytes, void** ptr, void* ipc_handle) {
  using namespace nvb::api_detail;
  g_last_error[0] = 0;
  if (!ptr || !ipc_handle || bytes == 0) return fail("invalid peer buffer arguments");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaMalloc(peer buffer)");
  e = cudaMemset(*ptr, 0, bytes);  // flags start at epoch 0
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return cuda_status(e, "peer buffer set-up");
  }
  return 0;
}

extern "C" int nvb_peer_buffer_open(const void* ipc_handle, void** ptr) {
  using namespace nvb::api_detail;
  g_last_error[0] = 0;
  if (!ptr || !ipc_handle) return fail("invalid peer buffer arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

extern "C" int nvb_peer_buffer_close(void* ptr) {
  using namespace nvb::api_detail;
  g_last_error[0] = 0;
  return cuda_status(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

extern "C" int nvb_peer_buffer_free(void* ptr) {
  using namespace nvb::api_detail;
  g_last_error[0] = 0;
  return cuda_status(cudaFree(ptr), "cudaFree(peer buffer)");
}

namespace nvb {
namespace gather_detail {

// combine_gather_kernel with W warps per item (combine_detail::combine_warps).
template <bool kBarrier>
cudaError_t launch_combine_gather(const cudaLaunchConfig_t& cfg, int w, const float* la, const float* oa,
                                  const __nv_bfloat16* lo, int rows, int qh, int splits, PeerPtrs peers, int world,
                                  int head_offset, int qh_total, unsigned int* counter, int rank) {
  switch (w) {
    case 1:
      return cudaLaunchKernelEx(&cfg, combine_gather_kernel<kBarrier, 1>, la, oa, lo, rows, qh, splits, peers, world,
                                head_offset, qh_total, counter, rank);
    case 2:
      return cudaLaunchKernelEx(&cfg, combine_gather_kernel<kBarrier, 2>, la, oa, lo, rows, qh, splits, peers, world,
                                head_offset, qh_total, counter, rank);
    case 4:
      return cudaLaunchKernelEx(&cfg, combine_gather_kernel<kBarrier, 4>, la, oa, lo, rows, qh, splits, peers, world,
                                head_offset, qh_total, counter, rank);
    default:
      return cudaLaunchKernelEx(&cfg, combine_gather_kernel<kBarrier, 8>, la, oa, lo, rows, qh, splits, peers, world,
                                head_offset, qh_total, counter, rank);
  }
}

int gather_impl(void* stream, const void* q, const void* k, const void* v, void* out_local, const int* cu_q,
                const int* kv_lens, const int* block_table, int batch, int max_k, int q_heads, int kv_heads,
                int block_size, int table_stride, int num_blocks, int num_splits, float* lse_accum, float* out_accum,
                void* const* out0, void* const* out1, unsigned int* const* peer_flag, int world, int rank,
                unsigned int epoch) {
  using namespace nvb::api_detail;
  g_last_error[0] = 0;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || !out0 || !peer_flag || batch <= 0 ||
      q_heads <= 0)
    return fail("invalid gather arguments (world 1..%d, rank in [0, world))", kMaxRanks);
  PeerPtrs peers{};
  for (int p = 0; p < world; ++p) {
    for (int set = 0; set < (out1 ? 2 : 1); ++set) {
      void* o = set ? out1[p] : out0[p];
      if (!o || (reinterpret_cast<uintptr_t>(o) & 15))
        return fail("peer %d: outputs must be non-null and 16-byte aligned", p);
      peers.out[set][p] = static_cast<__nv_bfloat16*>(o);
    }
    if (!peer_flag[p] || (reinterpret_cast<uintptr_t>(peer_flag[p]) & 3))
      return fail("peer %d: flags must be non-null and 4-byte aligned", p);
    peers.flag[p] = peer_flag[p];
  }
  unsigned int* counter = out1 ? peer_flag[rank] + world : nullptr;
  const bool partials = num_splits > 1 && block_size % 128 == 0;
  const int rc = paged_fwd_impl(stream, q, k, v, out_local, cu_q, kv_lens, block_table, batch, batch, 1, max_k,
                                q_heads, kv_heads, block_size, table_stride, num_splits, nullptr, lse_accum,
                                out_accum, num_blocks, true, !partials);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long items = (long long)batch * q_heads;
  // Both kernels are programmatic dependents of the kernel before them on the
  // stream, so each launch overlaps its predecessor's tail; each waits in
  // griddepcontrol.wait for the predecessor to complete.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  const int splits = partials ? num_splits : 1;
  const int w = combine_detail::combine_warps(splits);
  const int per_cta = combine_detail::kCombineThreads / 32 / w;  // items a CTA combines
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned((items + per_cta - 1) / per_cta));
  cfg.blockDim = dim3(combine_detail::kCombineThreads);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const float* la = static_cast<const float*>(lse_accum);
  const float* oa = static_cast<const float*>(out_accum);
  const __nv_bfloat16* lo = static_cast<const __nv_bfloat16*>(out_local);
  if (counter) {
    // Counter form: the combine's last CTA runs the epoch exchange.
    const cudaError_t e = launch_combine_gather<true>(cfg, w, la, oa, lo, batch, q_heads, splits, peers, world,
                                                      rank * q_heads, world * q_heads, counter, rank);
    return cuda_status(e, "gather launch");
  }
  cudaError_t e = launch_combine_gather<false>(cfg, w, la, oa, lo, batch, q_heads, splits, peers, world,
                                               rank * q_heads, world * q_heads, counter, rank);
  if (e == cudaSuccess) {
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    e = cudaLaunchKernelEx(&cfg, gather_barrier_kernel, peers, world, rank, epoch, counter);
  }
  return cuda_status(e, "gather launch");
}

}  // namespace gather_detail
}  // namespace nvb

extern "C" int nvb_paged_decode_gather(void* stream, const void* q, const void* k, const void* v, void* out_local,
                                       const int* cu_q, const int* kv_lens, const int* block_table, int batch,
                                       int max_k, int q_heads, int kv_heads, int block_size, int table_stride,
                                       int num_blocks, int num_splits, float* lse_accum, float* out_accum,
                                       void* const* peer_out, unsigned int* const* peer_flag, int world, int rank,
                                       unsigned int epoch) {
  return nvb::gather_detail::gather_impl(stream, q, k, v, out_local, cu_q, kv_lens, block_table, batch, max_k,
                                         q_heads, kv_heads, block_size, table_stride, num_blocks, num_splits,
                                         lse_accum, out_accum, peer_out, nullptr, peer_flag, world, rank, epoch);
}

extern "C" int nvb_paged_decode_gather_capturable(void* stream, const void* q, const void* k, const void* v,
                                                  void* out_local, const int* cu_q, const int* kv_lens,
                                                  const int* block_table, int batch, int max_k, int q_heads,
                                                  int kv_heads, int block_size, int table_stride, int num_blocks,
                                                  int num_splits, float* lse_accum, float* out_accum,
                                                  void* const* peer_out0, void* const* peer_out1,
                                                  unsigned int* const* peer_flag, int world, int rank) {
  using namespace nvb::api_detail;
  if (!peer_out1) {
    g_last_error[0] = 0;
    return fail("the capturable gather needs two output sets");
  }
  return nvb::gather_detail::gather_impl(stream, q, k, v, out_local, cu_q, kv_lens, block_table, batch, max_k,
                                         q_heads, kv_heads, block_size, table_stride, num_blocks, num_splits,
                                         lse_accum, out_accum, peer_out0, peer_out1, peer_flag, world, rank, 0u);
}
