"""Many caches from one host thread: every launch reads its own K and V.

The library keeps a per-thread cache of TMA descriptors keyed by base
pointer and geometry. An engine with L layers addresses 2L caches in decode
and again in prefill (plus query buffers), far more than any small cache
holds, and each launch looks up two or three descriptors in a row. These
tests interleave launches over 48 distinct K/V buffers in an order that mixes
cache hits and misses, pair each K with a different V, and check every
output against the FP32 oracle, for decode and for prefill.
"""
import random

import pytest
import torch

from conftest import as_f32, assert_close, bits

pytestmark = pytest.mark.gpu

N_BUF = 48


def _buffers(nvb, q_lens, kv_lens, seed):
    W = nvb.workloads
    base = W.paged_case(kv_lens, q_lens, q_heads=8, kv_heads=4, seed=seed, scale=1.0)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    bufs = [(torch.randn(base.k.shape, generator=g, device="cuda")).bfloat16() for _ in range(N_BUF)]
    return base, bufs


def _oracle(oracle, case, k, v):
    out, _ = oracle.attention_varlen(bits(case.q), bits(k), bits(v), case.cu_q.cpu().numpy(),
                                     case.kv_lens.cpu().numpy(), case.block_table.cpu().numpy(), qh=case.q_heads,
                                     kvh=case.kv_heads, bs=case.block_size, blocks=case.num_blocks,
                                     stride=case.table_stride, threads=8)
    return out


@pytest.mark.parametrize("mode", ["decode", "prefill"])
def test_interleaved_launches_over_many_caches(nvb, oracle, mode):
    if mode == "decode":
        base, bufs = _buffers(nvb, None, [300, 517], seed=21)
        max_q, splits = 1, 3
    else:
        base, bufs = _buffers(nvb, [200, 64], [300, 517], seed=23)
        max_q, splits = 200, 1
    b, qh = base.batch, base.q_heads
    la, oa = nvb.splitkv_scratch(splits, b, qh, "cuda") if splits > 1 else (None, None)
    rng = random.Random(7)
    # a sequence of (k index, v index) that revisits buffers irregularly
    order = [(i, (i * 7 + 3) % N_BUF) for i in range(N_BUF)]
    order += [(rng.randrange(N_BUF), rng.randrange(N_BUF)) for _ in range(120)]
    order += [(i % 5, (i + 1) % 5) for i in range(20)]
    outs = []
    for ki, vi in order:
        out = torch.empty_like(base.q)
        nvb.paged_fwd(base.q, bufs[ki], bufs[vi], out, base.cu_q, base.kv_lens, base.block_table, batch=b,
                      max_q=max_q, max_k=int(base.kv_lens.max()), q_heads=qh, kv_heads=base.kv_heads,
                      block_size=base.block_size, table_stride=base.table_stride, num_blocks=base.num_blocks,
                      num_splits=splits, lse_accum=la, out_accum=oa)
        outs.append(out)
    torch.cuda.synchronize()
    checked = {}
    for (ki, vi), out in zip(order, outs):
        key = (ki, vi)
        if key not in checked:
            checked[key] = _oracle(oracle, base, bufs[ki], bufs[vi])
        assert_close(as_f32(out), checked[key], 2e-2, 2e-3, f"{mode} launch with K {ki}, V {vi}")
    assert nvb.device_error() == 0
