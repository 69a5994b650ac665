"""One small decode-layer step on cuda:0, checked against the CPU oracle.

Used by __graft_entry__.smoke(): the fused Q/K-norm + RoPE + KV store writes
each sequence's new token into the paged cache, then split-KV decode
attention reads the whole context. The oracle repeats both steps on the host.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]


def run(nvb) -> None:
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle  # the checker

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    W = nvb.workloads
    qh, kvh, bs = 16, 8, 256
    lens = [33, 300, 700, 1]  # contexts after this step's token
    case = W.paged_case(lens, q_heads=qh, kv_heads=kvh, block_size=bs, seed=3, device="cuda")
    b = case.batch
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = torch.randn(b, qh + 2 * kvh, 128, generator=g, device="cuda").bfloat16()
    qw = (1 + 0.02 * torch.randn(128, generator=g, device="cuda")).bfloat16()
    kw = (1 + 0.02 * torch.randn(128, generator=g, device="cuda")).bfloat16()
    positions = (case.kv_lens - 1).to(torch.int32)
    table = case.block_table.cpu()
    slots = torch.tensor([int(table[i, p // bs]) * bs + p % bs for i, p in enumerate(positions.tolist())],
                         dtype=torch.int32, device="cuda")
    rope = torch.empty(4096, 128, dtype=torch.float32, device="cuda")
    nvb.rope_cache(rope, 4096, 128, 1e6)

    def host_bits(t):
        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).copy()

    k0, v0 = host_bits(case.k), host_bits(case.v)
    nvb.qkv_rope_cached(qkv, qw, kw, positions, slots, case.q, case.k, case.v, rows=b, q_heads=qh, kv_heads=kvh,
                        head_dim=128, block_size=bs, num_blocks=case.num_blocks, eps=1e-6, rope_cache=rope,
                        max_positions=4096)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    splits = nvb.num_splits(b, qh, kvh, 4096, sms)
    out = torch.empty_like(case.q)
    lse = torch.empty(b, qh, 1, dtype=torch.float32, device="cuda")
    la, oa = nvb.splitkv_scratch(splits, b, qh, "cuda") if splits > 1 else (None, None)
    nvb.paged_fwd(case.q, case.k, case.v, out, case.cu_q, case.kv_lens, case.block_table, batch=b, max_q=1,
                  max_k=4096 if case.table_stride * bs >= 4096 else case.table_stride * bs, q_heads=qh,
                  kv_heads=kvh, block_size=bs, table_stride=case.table_stride, num_blocks=case.num_blocks,
                  num_splits=splits, lse=lse, lse_accum=la, out_accum=oa)
    torch.cuda.synchronize()

    qo = np.zeros((b, qh, 128), np.uint16)
    oracle.qkv_rope(host_bits(qkv), host_bits(qw), host_bits(kw), positions.cpu().numpy(), slots.cpu().numpy(), qo,
                    k0, v0, qh=qh, kvh=kvh, dim=128, bs=bs, blocks=case.num_blocks, eps=1e-6,
                    rope_cache=rope.cpu().numpy(), max_positions=4096)
    # The decode check uses the GPU's Q and caches (the fused kernel is
    # compared separately, within one BF16 rounding step).
    qf = oracle.bits_to_f32(qo)
    if not np.abs(case.q.float().cpu().numpy() - qf).max() <= 0.0625:
        raise AssertionError("fused store Q differs from the oracle")
    ref, ref_lse = oracle.attention_varlen(host_bits(case.q), host_bits(case.k), host_bits(case.v),
                                           case.cu_q.cpu().numpy(), case.kv_lens.cpu().numpy(),
                                           case.block_table.cpu().numpy(), qh=qh, kvh=kvh, bs=bs,
                                           blocks=case.num_blocks, stride=case.table_stride)
    err = np.abs(out.float().cpu().numpy() - ref)
    if not (np.isfinite(err).all() and err.max() <= 2e-2 and err.mean() <= 2e-3):
        raise AssertionError(f"smoke decode mismatch: max-abs {err.max():.3g}, mean-abs {err.mean():.3g}")
    lerr = np.abs(lse.cpu().numpy() - ref_lse).max()
    if not lerr <= 1e-3:
        raise AssertionError(f"smoke lse mismatch: {lerr:.3g}")
    print(f"smoke ok: splits={splits} max-abs {err.max():.3g} mean-abs {err.mean():.3g} lse {lerr:.3g}")
