"""Multi-GPU decode sharding for the paged attention path.

Two partitions of the work, one process per GPU over torch.distributed:

* by sequence (configuration 3, engine replicas of configuration 4): each
  rank decodes its own sequences against its own cache; there is no
  collective on the data path (`sequence_shard`).
* by kv head (configuration 5, long context): rank r owns kv heads
  [r*kvh_local, (r+1)*kvh_local) of every sequence and the query heads of
  their GQA groups; its cache holds only those kv heads. Each rank runs the
  split-KV decode on its heads and every rank needs the whole
  [batch, q_heads, 128] output (`KvHeadShardedDecode`). The transfer is
  batch * q_heads * 256 B (8 KiB per rank at 4 x 64 heads), so a separate
  collective is launch-latency bound. The default (`fused=True`) stores each
  combined result straight into every rank's output from the combine kernel
  (peer stores over NVLink into CUDA IPC buffers, then an epoch-flag barrier
  whose epoch lives in device memory: nvb_paged_decode_gather_capturable), so
  a whole step can be captured in a CUDA graph once and replayed;
  `fused=False` keeps the NCCL all-gather.

The reference is single-GPU (its README: no NCCL, MPI or tensor
parallelism); this module is the B200 build's own.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    kv_heads: int          # total kv heads
    q_heads: int           # total query heads

    def __post_init__(self):
        if self.kv_heads % self.world or self.q_heads % self.kv_heads:
            raise ValueError(f"{self.kv_heads} kv heads / {self.q_heads} q heads do not shard over {self.world} ranks")

    @property
    def kv_local(self) -> int:
        return self.kv_heads // self.world

    @property
    def q_local(self) -> int:
        return self.q_heads // self.world

    @property
    def kv_range(self):
        return range(self.rank * self.kv_local, (self.rank + 1) * self.kv_local)

    @property
    def q_range(self):
        return range(self.rank * self.q_local, (self.rank + 1) * self.q_local)


def sequence_shard(batch: int, rank: int, world: int):
    """Contiguous sequence range of `rank` (sizes differ by at most one)."""
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def gather_heads(local_out, shard: HeadShard, group=None):
    """All-gathers per-rank outputs [batch, q_local, D] into [batch, q_heads, D]
    with query heads in global order."""
    import torch
    import torch.distributed as dist

    b, ql, d = local_out.shape
    buf = torch.empty(shard.world * b * ql * d, dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(buf, local_out.contiguous().view(-1), group=group)
    return buf.view(shard.world, b, ql, d).permute(1, 0, 2, 3).reshape(b, shard.world * ql, d)


def exchange_peer_buffers(nvb, shard: HeadShard, ptr, handle, group=None):
    """All-gathers the ranks' IPC handles and maps the peers' buffers:
    returns every rank's base pointer in rank order (this rank's own `ptr`
    at its index)."""
    import torch.distributed as dist

    handles = [handle]
    if shard.world > 1:
        handles = [None] * shard.world
        dist.all_gather_object(handles, handle, group=group)
    return [ptr if r == shard.rank else nvb.peer_buffer_open(h) for r, h in enumerate(handles)]


class _DeviceArray:
    """A torch view of device memory the library allocated (CUDA array
    interface)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3, "strides": None}


class KvHeadShardedDecode:
    """Decode over a kv-head-sharded paged cache, then every rank gets the
    whole output. `k_local` / `v_local` are this rank's caches
    [num_blocks, block_size, kv_local, 128]; `q_local` is
    [batch, q_local, 128] (the query heads of this rank's kv heads).
    fused=True (default): combine and all-gather in one kernel through peer
    memory; the returned tensor is one of two output buffers used in turn.
    Read it (or enqueue its readers on the current stream) before this
    rank's next call: a peer stores the step after that into the same
    buffer as soon as this rank's next step has signalled. `capture` records one such
    step in a CUDA graph and `replay` runs it (every rank must call and
    replay in the same order). fused=False: NCCL all-gather.
    Call close() before destroying the process group."""

    FLAG_BYTES = 256

    def __init__(self, nvb, shard: HeadShard, *, batch, block_size, table_stride, num_blocks, max_k, device,
                 num_splits=None, group=None, fused=True):
        import torch

        self.nvb, self.shard, self.group, self.fused = nvb, shard, group, fused
        self.batch, self.block_size, self.table_stride = batch, block_size, table_stride
        self.num_blocks, self.max_k = num_blocks, max_k
        sms = torch.cuda.get_device_properties(device).multi_processor_count
        self.splits = num_splits or nvb.num_splits(batch, shard.q_local, shard.kv_local, max_k, sms)
        self.out_local = torch.empty(batch, shard.q_local, 128, dtype=torch.bfloat16, device=device)
        self.lse = torch.empty(batch, shard.q_local, 1, dtype=torch.float32, device=device)
        self.la, self.oa = (nvb.splitkv_scratch(self.splits, batch, shard.q_local, device) if self.splits > 1
                            else (None, None))
        self.epoch = 0
        self._own = None
        self._peers = []
        if fused:
            self._setup_peers(device)

    def _setup_peers(self, device):
        """One IPC-shared device buffer per rank: flags, then two outputs."""
        import torch

        out_elems = self.batch * self.shard.q_heads * 128
        self.out_bytes = (out_elems * 2 + 255) // 256 * 256
        with torch.cuda.device(device):
            ptr, handle = self.nvb.peer_buffer_create(self.FLAG_BYTES + 2 * self.out_bytes)
            self._own = ptr
            bases = exchange_peer_buffers(self.nvb, self.shard, ptr, handle, self.group)
            self._peers = [b for r, b in enumerate(bases) if r != self.shard.rank]
        self.flag_ptrs = bases
        self.out_ptrs = [[b + self.FLAG_BYTES + i * self.out_bytes for b in bases] for i in range(2)]
        shape = (self.batch, self.shard.q_heads, 128)
        self.views = [torch.as_tensor(_DeviceArray(ptr + self.FLAG_BYTES + i * self.out_bytes, shape, "<i2"),
                                      device=device).view(torch.bfloat16) for i in range(2)]

    def close(self):
        """Unmaps the peers' buffers and frees this rank's (fused mode)."""
        for p in self._peers:
            self.nvb.peer_buffer_close(p)
        self._peers = []
        if self._own is not None:
            self.views = []
            self.nvb.peer_buffer_free(self._own)
            self._own = None

    def local(self, q_local, k_local, v_local, cu_q, kv_lens, block_table, check=True):
        self.nvb.paged_fwd(q_local, k_local, v_local, self.out_local, cu_q, kv_lens, block_table, batch=self.batch,
                           max_q=1, max_k=self.max_k, q_heads=self.shard.q_local, kv_heads=self.shard.kv_local,
                           block_size=self.block_size, table_stride=self.table_stride, num_blocks=self.num_blocks,
                           num_splits=self.splits, lse=self.lse, lse_accum=self.la, out_accum=self.oa, check=check)
        return self.out_local

    def __call__(self, q_local, k_local, v_local, cu_q, kv_lens, block_table, check=True):
        if not self.fused:
            self.local(q_local, k_local, v_local, cu_q, kv_lens, block_table, check)
            return gather_heads(self.out_local, self.shard, self.group)
        self._fused_step(q_local, k_local, v_local, cu_q, kv_lens, block_table, check)
        self.epoch += 1
        return self.views[self.epoch & 1]

    def _fused_step(self, q_local, k_local, v_local, cu_q, kv_lens, block_table, check):
        # The step's epoch is the device counter + 1 (advanced by the step
        # itself); self.epoch mirrors it on the host to name the output set.
        self.nvb.paged_decode_gather_capturable(
            q_local, k_local, v_local, self.out_local, cu_q, kv_lens, block_table, batch=self.batch,
            max_k=self.max_k, q_heads=self.shard.q_local, kv_heads=self.shard.kv_local, block_size=self.block_size,
            table_stride=self.table_stride, num_blocks=self.num_blocks, num_splits=self.splits, lse_accum=self.la,
            out_accum=self.oa, peer_out0=self.out_ptrs[0], peer_out1=self.out_ptrs[1], peer_flag=self.flag_ptrs,
            rank=self.shard.rank, check=check)

    def capture(self, q_local, k_local, v_local, cu_q, kv_lens, block_table):
        """A CUDA graph of one fused step on these inputs (nothing runs while
        capturing). Call the step eagerly once before, so the library has
        set up its kernels and descriptors."""
        import torch

        if not self.fused:
            raise ValueError("capture needs the fused gather")
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self._fused_step(q_local, k_local, v_local, cu_q, kv_lens, block_table, True)
        return graph

    def replay(self, graph):
        """Runs a captured step; returns this step's output set."""
        graph.replay()
        self.epoch += 1
        return self.views[self.epoch & 1]
