"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference publishes no dataset for this path; its configurations are
shapes plus value distributions (q/K/V ~ N(0,1)*scale, context lengths
uniform in a range, a permuted page table), so these generators stand in for
them. Page ids are a seeded permutation of the physical pages (the
reference's own BlockPool is deterministic; the benchmark asks for a
shuffled table).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

HEAD_DIM = 128


@dataclass
class PagedCase:
    q: torch.Tensor            # [total_q, qh, 128] bf16
    k: torch.Tensor            # [num_blocks, block_size, kvh, 128] bf16
    v: torch.Tensor
    block_table: torch.Tensor  # [batch, table_stride] int32, -1 padded
    kv_lens: torch.Tensor      # [batch] int32
    cu_q: torch.Tensor         # [batch + 1] int32
    q_heads: int
    kv_heads: int
    block_size: int
    table_stride: int
    num_blocks: int

    @property
    def batch(self) -> int:
        return self.kv_lens.numel()

    @property
    def max_q(self) -> int:
        return int((self.cu_q[1:] - self.cu_q[:-1]).max().item())

    def kv_bytes(self) -> int:
        """Algorithmic K+V bytes read: 512 B per token per kv head."""
        return int(self.kv_lens.sum().item()) * self.kv_heads * HEAD_DIM * 2 * 2


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def paged_case(kv_lens, q_lens=None, *, q_heads, kv_heads, block_size=256, seed=0, scale=0.5, device="cuda",
               spare_blocks=0, shuffle=True, table_stride=None) -> PagedCase:
    """Builds a paged KV cache holding `kv_lens[b]` tokens for each sequence,
    with queries q_lens[b] (default 1: decode). Values ~ N(0, 1) * scale."""
    kv_lens = [int(x) for x in kv_lens]
    q_lens = [1] * len(kv_lens) if q_lens is None else [int(x) for x in q_lens]
    pages = [(n + block_size - 1) // block_size for n in kv_lens]
    num_blocks = sum(pages) + spare_blocks
    stride = table_stride or max(pages)
    g_cpu = _gen("cpu", seed)
    perm = torch.randperm(num_blocks, generator=g_cpu) if shuffle else torch.arange(num_blocks)
    table = torch.full((len(kv_lens), stride), -1, dtype=torch.int32)
    cursor = 0
    for b, n in enumerate(pages):
        table[b, :n] = perm[cursor:cursor + n].to(torch.int32)
        cursor += n
    g = _gen(device, seed + 1)
    total_q = sum(q_lens)
    q = (torch.randn(total_q, q_heads, HEAD_DIM, generator=g, device=device) * scale).to(torch.bfloat16)
    k = (torch.randn(num_blocks, block_size, kv_heads, HEAD_DIM, generator=g, device=device) * scale).to(
        torch.bfloat16)
    v = (torch.randn(num_blocks, block_size, kv_heads, HEAD_DIM, generator=g, device=device) * scale).to(
        torch.bfloat16)
    cu = torch.zeros(len(q_lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(q_lens, dtype=torch.int32), 0)
    return PagedCase(q=q, k=k, v=v, block_table=table.to(device), kv_lens=torch.tensor(kv_lens, dtype=torch.int32,
                     device=device), cu_q=cu.to(device), q_heads=q_heads, kv_heads=kv_heads, block_size=block_size,
                     table_stride=stride, num_blocks=num_blocks)


def uniform_lengths(n, lo, hi, seed):
    g = _gen("cpu", seed)
    return torch.randint(lo, hi + 1, (n,), generator=g).tolist()


# Benchmark configurations (shapes from the reference's benchmark plan).
def config1_decode(device="cuda", seed=0):
    """Qwen3-0.6B layer: 16q/8kv, batch 8, ctx ~ U[128, 1024]."""
    return paged_case(uniform_lengths(8, 128, 1024, seed), q_heads=16, kv_heads=8, seed=seed, device=device)


def config3_decode(device="cuda", seed=0, batch=256, ctx=4096):
    """Qwen3-8B attention shape: 32q/8kv, batch 256, ctx 4096."""
    return paged_case([ctx] * batch, q_heads=32, kv_heads=8, seed=seed, device=device)


def config5_decode(device="cuda", seed=0, batch=4, ctx=32768, kv_heads=8, q_heads=64):
    """Qwen3-32B attention shape: 64q/8kv, batch 4, ctx 32768."""
    return paged_case([ctx] * batch, q_heads=q_heads, kv_heads=kv_heads, seed=seed, device=device)


def config2_prefill(device="cuda", seed=0, n=32, lo=64, hi=2048):
    """Qwen3-0.6B varlen causal prefill: 32 prompts with L ~ U[64, 2048]."""
    lens = uniform_lengths(n, lo, hi, seed)
    return paged_case(lens, lens, q_heads=16, kv_heads=8, seed=seed, device=device, scale=1.0)


def config2_chunked(device="cuda", seed=0, n=32, chunk=64):
    """Chunked prefill: a pre-filled prefix P ~ U[256, 2048], then one
    64-token chunk per sequence."""
    prefix = uniform_lengths(n, 256, 2048, seed)
    return paged_case([p + chunk for p in prefix], [chunk] * n, q_heads=16, kv_heads=8, seed=seed, device=device,
                      scale=1.0)


def prefill_flops(case: PagedCase) -> float:
    """Causal attention FLOPs counting only visible keys: 4 * 128 * qh per
    (query, visible key) pair."""
    total = 0
    cu = case.cu_q.tolist()
    lens = case.kv_lens.tolist()
    for b in range(case.batch):
        ql = cu[b + 1] - cu[b]
        kl = lens[b]
        # query i sees kl - ql + i + 1 keys
        total += ql * (kl - ql) + ql * (ql + 1) // 2
    return 4.0 * HEAD_DIM * case.q_heads * total
