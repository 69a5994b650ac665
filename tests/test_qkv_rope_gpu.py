"""Fused Q/K RMSNorm + RoPE + paged KV store on the GPU.

Parity bar: bit-identical to the reference's own kernel
(qkv_rope_kernel<CACHED>, kernels/kernels.cu:166-211, built from source into
oracle/_ref), within one BF16 rounding step of the CPU oracle, and an exact
slot scatter. Known answers follow src/gpu.rs:1246-1289 and 1330-1380.
"""
import math

import numpy as np
import pytest
import torch

from conftest import as_f32, assert_close, bits

pytestmark = pytest.mark.gpu

QH, KVH, DIM, BS, BLOCKS, MAXPOS = 16, 8, 128, 256, 6, 4096
EPS, THETA = 1e-6, 1e6


def _inputs(rows, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qkv = torch.randn(rows, QH + 2 * KVH, DIM, generator=g, device="cuda").bfloat16()
    qw = (1 + 0.02 * torch.randn(DIM, generator=g, device="cuda")).bfloat16()
    kw = (1 + 0.02 * torch.randn(DIM, generator=g, device="cuda")).bfloat16()
    gc = torch.Generator().manual_seed(seed)
    positions = torch.randint(0, MAXPOS, (rows,), generator=gc, dtype=torch.int32)
    slots = torch.randperm(BS * BLOCKS, generator=gc)[:rows].to(torch.int32)
    # edge cases: out-of-range positions (cos 1, sin 0) and skipped slots
    for i, val in enumerate((0, MAXPOS - 1, -5, MAXPOS + 7)):
        if i < rows:
            positions[i] = val
    for i, val in ((4, -1), (5, BS * BLOCKS)):
        if i < rows:
            slots[i] = val
    return qkv, qw, kw, positions.cuda(), slots.cuda()


def _caches(seed):
    g = torch.Generator(device="cuda").manual_seed(seed + 99)
    shape = (BLOCKS, BS, KVH, DIM)
    return torch.randn(shape, generator=g, device="cuda").bfloat16(), torch.randn(shape, generator=g,
                                                                                  device="cuda").bfloat16()


def _run_nvb(nvb, qkv, qw, kw, pos, slots, table, rows):
    qout = torch.zeros(rows, QH, DIM, dtype=torch.bfloat16, device="cuda")
    kc, vc = _caches(1)
    nvb.qkv_rope_cached(qkv, qw, kw, pos, slots, qout, kc, vc, rows=rows, q_heads=QH, kv_heads=KVH, head_dim=DIM,
                        block_size=BS, num_blocks=BLOCKS, eps=EPS, rope_cache=table, max_positions=MAXPOS)
    torch.cuda.synchronize()
    return qout, kc, vc


def test_rope_table_bit_exact_vs_reference_kernel(nvb, ref_native):
    mine = torch.empty(MAXPOS, DIM, dtype=torch.float32, device="cuda")
    ref = torch.empty_like(mine)
    nvb.rope_cache(mine, MAXPOS, DIM, THETA)
    torch.cuda.synchronize()
    ref_native.call("nv_rope_cache", ref, MAXPOS, DIM, THETA)
    assert torch.equal(mine.view(torch.int32), ref.view(torch.int32))


def test_rope_table_matches_cpu_oracle(nvb, oracle):
    mine = torch.empty(MAXPOS, DIM, dtype=torch.float32, device="cuda")
    nvb.rope_cache(mine, MAXPOS, DIM, THETA)
    torch.cuda.synchronize()
    expect = oracle.rope_cache(MAXPOS, DIM, THETA)
    # CUDA's powf/sincosf against the C library's: a few ulp, amplified by
    # the angle (up to 4095 rad) for the table's fastest pairs.
    assert_close(mine.cpu().numpy(), expect, 2e-3, 1e-5, "rope table")


@pytest.mark.parametrize("rows", [1, 37, 1024])
def test_fused_store_bit_exact_vs_reference_kernel(nvb, ref_native, rows):
    qkv, qw, kw, pos, slots = _inputs(rows, seed=rows)
    table = torch.empty(MAXPOS, DIM, dtype=torch.float32, device="cuda")
    nvb.rope_cache(table, MAXPOS, DIM, THETA)
    qout, kc, vc = _run_nvb(nvb, qkv, qw, kw, pos, slots, table, rows)
    rq = torch.zeros_like(qout)
    rk, rv = _caches(1)
    ref_native.call("nv_qkv_rope_cached", qkv, qw, kw, pos, slots, rq, rk, rv, rows, QH, KVH, DIM, BS, BLOCKS, EPS,
                    table, MAXPOS)
    assert torch.equal(qout.view(torch.int16), rq.view(torch.int16)), "Q differs from the reference kernel"
    assert torch.equal(kc.view(torch.int16), rk.view(torch.int16)), "K cache differs from the reference kernel"
    assert torch.equal(vc.view(torch.int16), rv.view(torch.int16)), "V cache differs from the reference kernel"


def test_direct_rope_bit_exact_vs_reference_kernel(nvb, ref_native):
    rows = 64
    qkv, qw, kw, pos, slots = _inputs(rows, seed=5)
    qout = torch.zeros(rows, QH, DIM, dtype=torch.bfloat16, device="cuda")
    kc, vc = _caches(2)
    nvb.qkv_rope(qkv, qw, kw, pos, slots, qout, kc, vc, rows=rows, q_heads=QH, kv_heads=KVH, head_dim=DIM,
                 block_size=BS, num_blocks=BLOCKS, eps=EPS, theta=THETA)
    torch.cuda.synchronize()
    rq = torch.zeros_like(qout)
    rk, rv = _caches(2)
    ref_native.call("nv_qkv_rope", qkv, qw, kw, pos, slots, rq, rk, rv, rows, QH, KVH, DIM, BS, BLOCKS, EPS, THETA)
    assert torch.equal(qout.view(torch.int16), rq.view(torch.int16))
    assert torch.equal(kc.view(torch.int16), rk.view(torch.int16))
    assert torch.equal(vc.view(torch.int16), rv.view(torch.int16))


def test_fused_store_matches_cpu_oracle_and_scatter_is_exact(nvb, oracle):
    rows = 200
    qkv, qw, kw, pos, slots = _inputs(rows, seed=11)
    table = torch.empty(MAXPOS, DIM, dtype=torch.float32, device="cuda")
    nvb.rope_cache(table, MAXPOS, DIM, THETA)
    qout, kc, vc = _run_nvb(nvb, qkv, qw, kw, pos, slots, table, rows)
    kc0, vc0 = _caches(1)
    oq = np.zeros((rows, QH, DIM), np.uint16)
    ok, ov = bits(kc0).copy(), bits(vc0).copy()
    oracle.qkv_rope(bits(qkv), bits(qw), bits(kw), pos.cpu().numpy(), slots.cpu().numpy(), oq, ok, ov, qh=QH,
                    kvh=KVH, dim=DIM, bs=BS, blocks=BLOCKS, eps=EPS, rope_cache=table.cpu().numpy(),
                    max_positions=MAXPOS)
    # V is a copy: exact, and only valid slots change (integer scatter).
    assert np.array_equal(bits(vc), ov)
    touched = np.zeros(BS * BLOCKS, bool)
    s = slots.cpu().numpy()
    touched[s[(s >= 0) & (s < BS * BLOCKS)]] = True
    kflat, k0 = bits(kc).reshape(BS * BLOCKS, -1), bits(kc0).reshape(BS * BLOCKS, -1)
    assert np.array_equal(kflat[~touched], k0[~touched]), "untouched K slots changed"
    # Q and rotated K: the CPU's 1/sqrtf may differ from rsqrtf by an ulp,
    # which can move a BF16 rounding by one step.
    assert_close(as_f32(qout), oracle.bits_to_f32(oq), 0.0625, 1e-3, "Q vs oracle")
    assert_close(oracle.bits_to_f32(kflat[touched]), oracle.bits_to_f32(ok.reshape(BS * BLOCKS, -1)[touched]),
                 0.0625, 1e-3, "K vs oracle")


def test_known_answers_all_ones(nvb):
    # src/gpu.rs:1364-1378 at head_dim 128: all-ones input, positions 0..2.
    rows = 3
    qkv = torch.ones(rows, QH + 2 * KVH, DIM, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(DIM, dtype=torch.bfloat16, device="cuda")
    pos = torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda")
    slots = torch.tensor([2, 3, 0], dtype=torch.int32, device="cuda")
    table = torch.empty(MAXPOS, DIM, dtype=torch.float32, device="cuda")
    nvb.rope_cache(table, MAXPOS, DIM, THETA)
    qout = torch.zeros(rows, QH, DIM, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(BLOCKS, BS, KVH, DIM, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    nvb.qkv_rope_cached(qkv, w, w, pos, slots, qout, kc, vc, rows=rows, q_heads=QH, kv_heads=KVH, head_dim=DIM,
                        block_size=BS, num_blocks=BLOCKS, eps=EPS, rope_cache=table, max_positions=MAXPOS)
    torch.cuda.synchronize()
    q = as_f32(qout)
    assert np.all(np.abs(q[0] - 1.0) < 0.01)
    assert abs(q[1, 0, 0] - (math.cos(1.0) - math.sin(1.0))) < 0.008
    assert as_f32(vc).reshape(-1, KVH, DIM)[2, 0, 0] == 1.0


def test_cached_matches_direct_at_context_boundary(nvb):
    # src/gpu.rs:1246-1289: byte equality at positions 0, 1, 350, 4095.
    rows = 4
    idx = torch.arange(rows * (QH + 2 * KVH) * DIM, device="cuda")
    qkv = (((idx * 17) % 37).float() - 18.0).div(8.0).bfloat16().view(rows, QH + 2 * KVH, DIM)
    w = torch.ones(DIM, dtype=torch.bfloat16, device="cuda")
    pos = torch.tensor([0, 1, 350, 4095], dtype=torch.int32, device="cuda")
    slots = torch.tensor([0, 1, 2, 3], dtype=torch.int32, device="cuda")
    table = torch.empty(MAXPOS, DIM, dtype=torch.float32, device="cuda")
    nvb.rope_cache(table, MAXPOS, DIM, THETA)
    outs = []
    for cached in (False, True):
        qout = torch.zeros(rows, QH, DIM, dtype=torch.bfloat16, device="cuda")
        kc = torch.zeros(1, 4, KVH, DIM, dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        kw = dict(rows=rows, q_heads=QH, kv_heads=KVH, head_dim=DIM, block_size=4, num_blocks=1, eps=EPS)
        if cached:
            nvb.qkv_rope_cached(qkv, w, w, pos, slots, qout, kc, vc, rope_cache=table, max_positions=MAXPOS, **kw)
        else:
            nvb.qkv_rope(qkv, w, w, pos, slots, qout, kc, vc, theta=THETA, **kw)
        outs.append((qout, kc, vc))
    torch.cuda.synchronize()
    for a, b in zip(*outs):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_rejects_unsupported_head_dim(nvb):
    t = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    i = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(nvb.NvbError, match="head_dim 128"):
        nvb.qkv_rope(t, t, t, i, i, t, t, t, rows=1, q_heads=1, kv_heads=1, head_dim=64, block_size=1,
                     num_blocks=1, eps=EPS, theta=THETA)


@pytest.mark.parametrize("seed", range(8))
def test_fused_store_random_shapes_bit_exact_vs_reference_kernel(nvb, ref_native, seed):
    # Random head counts, row counts, input scales, table lengths, positions
    # (some before 0 or past the table) and slots (some outside the cache):
    # Q, the K cache and the V cache equal the reference kernel's bit for bit.
    rng = np.random.default_rng(4000 + seed)
    kvh = int(rng.choice([1, 2, 4, 8]))
    qh = kvh * int(rng.choice([1, 2, 4, 8]))
    rows = int(rng.integers(1, 600))
    bs, maxpos = 256, int(rng.integers(16, 4097))
    blocks = rows // bs + 2
    scale = float(rng.choice([0.05, 1.0, 8.0]))
    g = torch.Generator(device="cuda").manual_seed(seed)
    qkv = (torch.randn(rows, qh + 2 * kvh, DIM, generator=g, device="cuda") * scale).bfloat16()
    qw = (1 + 0.02 * torch.randn(DIM, generator=g, device="cuda")).bfloat16()
    kw = (1 + 0.02 * torch.randn(DIM, generator=g, device="cuda")).bfloat16()
    pos = torch.from_numpy(rng.integers(-3, maxpos + 20, size=rows).astype(np.int32)).cuda()
    slots_np = rng.permutation(bs * blocks + 8)[:rows].astype(np.int32) - 4
    slots = torch.from_numpy(slots_np).cuda()
    table = torch.empty(maxpos, DIM, dtype=torch.float32, device="cuda")
    nvb.rope_cache(table, maxpos, DIM, THETA)
    shape = (blocks, bs, kvh, DIM)
    kc0 = torch.randn(shape, generator=g, device="cuda").bfloat16()
    vc0 = torch.randn(shape, generator=g, device="cuda").bfloat16()
    qout, kc, vc = torch.zeros(rows, qh, DIM, dtype=torch.bfloat16, device="cuda"), kc0.clone(), vc0.clone()
    nvb.qkv_rope_cached(qkv, qw, kw, pos, slots, qout, kc, vc, rows=rows, q_heads=qh, kv_heads=kvh, head_dim=DIM,
                        block_size=bs, num_blocks=blocks, eps=EPS, rope_cache=table, max_positions=maxpos)
    rq, rk, rv = torch.zeros_like(qout), kc0.clone(), vc0.clone()
    ref_native.call("nv_qkv_rope_cached", qkv, qw, kw, pos, slots, rq, rk, rv, rows, qh, kvh, DIM, bs, blocks, EPS,
                    table, maxpos)
    torch.cuda.synchronize()
    what = f"seed {seed}: {rows} rows, {qh}q/{kvh}kv, scale {scale}, table {maxpos}"
    assert torch.equal(qout.view(torch.int16), rq.view(torch.int16)), f"Q differs ({what})"
    assert torch.equal(kc.view(torch.int16), rk.view(torch.int16)), f"K cache differs ({what})"
    assert torch.equal(vc.view(torch.int16), rv.view(torch.int16)), f"V cache differs ({what})"
