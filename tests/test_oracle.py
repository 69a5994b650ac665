"""Pins the CPU oracle against the reference's own known-answer tests.

 * src/gpu.rs:1330-1358  causal paged attention with reversed physical
   blocks, head_dim 32, block_size 2: row r averages values 1..r+1 exactly.
 * src/gpu.rs:1359-1378  fused norm + RoPE on all-ones input.
 * src/gpu.rs:1381-1471  the ragged GQA CPU check is itself an FP32 oracle;
   both of its cases are recomputed here with an independent numpy version.
 * kernels/flash_native/smoke.cu:57-81  causal suffix rule of the varlen form.
Golden fixtures produced by the reference's own kernels (tests/golden/) pin it
further when present.
"""
import math
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_reversed_blocks_exact_known_answer(oracle):
    rows, dim, qh, kvh, bs = 3, 32, 2, 1, 2
    q = np.zeros((rows, qh, dim), np.float32)
    v = np.zeros((2 * bs * kvh * dim,), np.float32)
    v[2 * dim:3 * dim] = 1.0  # physical block 1, slot 0 -> logical token 0
    v[3 * dim:4 * dim] = 2.0
    v[0:dim] = 3.0            # physical block 0, slot 0 -> logical token 2
    k = np.zeros_like(v)
    out = oracle.attention_native(oracle.bf16_bits(q), oracle.bf16_bits(k), oracle.bf16_bits(v), [0, 1, 2],
                                  [0, 0, 0], [1, 0], qh=qh, kvh=kvh, dim=dim, bs=bs, blocks=2, stride=2, batch=1,
                                  max_context=4)
    for r in range(rows):
        assert np.all(out[r] == 1.0 + 0.5 * r)


def _numpy_attention(q, k, v, pos, seq, table, qh, kvh, dim, bs, stride):
    out = np.zeros((len(pos), qh, dim), np.float64)
    for row in range(len(pos)):
        ctx = pos[row] + 1
        for h in range(qh):
            kh = h // (qh // kvh)
            idx = [((table[seq[row] * stride + t // bs] * bs + t % bs) * kvh + kh) for t in range(ctx)]
            K, V = k.reshape(-1, dim)[idx], v.reshape(-1, dim)[idx]
            s = K @ q[row, h] / math.sqrt(dim)
            p = np.exp(s - s.max())
            out[row, h] = p @ V / p.sum()
    return out


@pytest.mark.parametrize("dim,bs,pos,seq,table", [
    (32, 2, [0, 2, 1, 0], [0, 0, 1, 2], [3, 1, 0, 2, 2, -1]),
    (128, 256, [0, 255, 256, 510], [0, 0, 1, 1], [3, 1, 0, 2]),
])
def test_ragged_gqa_cases(oracle, dim, bs, pos, seq, table):
    rows, qh, kvh, blocks = 4, 4, 2, 4
    qv = ((np.arange(rows * qh * dim) * 7 % 19).astype(np.float32) - 9) * 0.125
    kv = ((np.arange(blocks * bs * kvh * dim) * 11 % 23).astype(np.float32) - 11) * 0.125
    vv = ((np.arange(blocks * bs * kvh * dim) * 3 % 13).astype(np.float32) - 6) * 0.125
    got = oracle.attention_native(oracle.bf16_bits(qv), oracle.bf16_bits(kv), oracle.bf16_bits(vv), pos, seq, table,
                                  qh=qh, kvh=kvh, dim=dim, bs=bs, blocks=blocks, stride=2, batch=len(table) // 2,
                                  max_context=max(pos) + 1)
    ref = _numpy_attention(qv.reshape(rows, qh, dim).astype(np.float64), kv.astype(np.float64),
                           vv.astype(np.float64), pos, seq, table, qh, kvh, dim, bs, 2)
    assert np.abs(got - ref).max() < 1e-5


def test_varlen_form_is_causal_suffix_and_matches_native_form(oracle):
    rng = np.random.default_rng(0)
    qh, kvh, bs, blocks, stride = 4, 2, 256, 6, 3
    qlens, klens = [3, 1, 5], [300, 17, 600]
    table = np.array([4, 0, -1, 2, -1, -1, 5, 1, 3], np.int32)
    total = sum(qlens)
    q = oracle.bf16_bits(rng.standard_normal((total, qh, 128)).astype(np.float32))
    k = oracle.bf16_bits(rng.standard_normal((blocks * bs * kvh * 128,)).astype(np.float32))
    v = oracle.bf16_bits(rng.standard_normal((blocks * bs * kvh * 128,)).astype(np.float32))
    cu = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    out, lse = oracle.attention_varlen(q, k, v, cu, klens, table, qh=qh, kvh=kvh, bs=bs, blocks=blocks,
                                       stride=stride)
    pos, seqs = [], []
    for b in range(3):
        for i in range(qlens[b]):
            pos.append(klens[b] - qlens[b] + i)
            seqs.append(b)
    nat = oracle.attention_native(q, k, v, pos, seqs, table, qh=qh, kvh=kvh, dim=128, bs=bs, blocks=blocks,
                                  stride=stride, batch=3, max_context=4096)
    assert np.array_equal(out, nat)
    assert np.all(np.isfinite(lse[0, :, :3])) and np.all(np.isneginf(lse[1, :, 1:]))


def test_fused_rope_known_answers(oracle):
    rows, qh, kvh, dim = 3, 2, 1, 32
    qkv = oracle.bf16_bits(np.ones((rows, qh + 2 * kvh, dim), np.float32))
    w = oracle.bf16_bits(np.ones(dim, np.float32))
    qout = np.zeros((rows, qh, dim), np.uint16)
    kc = np.zeros((2 * 2 * kvh * dim,), np.uint16)
    vc = np.zeros_like(kc)
    oracle.qkv_rope(qkv, w, w, [0, 1, 2], [2, 3, 0], qout, kc, vc, qh=qh, kvh=kvh, dim=dim, bs=2, blocks=2,
                    eps=1e-6, theta=1e6)
    q = oracle.bits_to_f32(qout)
    assert np.all(np.abs(q[0] - 1) < 0.01)
    assert abs(q[1, 0, 0] - (math.cos(1) - math.sin(1))) < 0.008
    assert oracle.bits_to_f32(vc)[0] == 1.0


def test_bf16_rounding_is_nearest_even(oracle):
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf], np.float32)
    b = oracle.bf16_bits(x)
    assert list(oracle.bits_to_f32(b)[:4]) == [1.0, 1.0, 1.015625, -2.5]
    assert np.isinf(oracle.bits_to_f32(b)[5])


def _golden_files():
    return sorted(GOLDEN.glob("*.npz"))


@pytest.mark.skipif(not _golden_files(), reason="no golden fixtures")
@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: p.stem)
def test_oracle_matches_reference_kernel_fixtures(oracle, path):
    """Fixtures written by tests/golden/make_golden.py from the reference's own
    CUDA kernels (oracle/_ref/libref_native.so) on a B200."""
    import golden_check

    golden_check.check(oracle, np.load(path, allow_pickle=False), path.stem)


def _from_bf16(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


@pytest.mark.parametrize("seed", range(12))
def test_varlen_random_shapes_match_numpy(oracle, seed):
    # The varlen oracle against an independent float64 numpy computation on
    # random shapes: query i of a q_len group sees keys [0, kv_len - q_len + i]
    # (src/model.rs:1170-1188) except those on an invalid (-1) page; LSE is the
    # natural log of the softmax denominator at scale 1/sqrt(128).
    rng = np.random.default_rng(seed)
    kvh = int(rng.choice([1, 2, 4]))
    qh = kvh * int(rng.choice([1, 2, 3, 4]))
    bs = int(rng.choice([16, 32, 256]))
    batch = int(rng.integers(1, 5))
    q_lens = rng.integers(1, 9, size=batch)
    kv_lens = q_lens + rng.integers(0, 300, size=batch)
    stride = int(max((kv_lens + bs - 1) // bs))
    blocks = batch * stride + 2
    table = rng.permutation(blocks)[:batch * stride].astype(np.int32).reshape(batch, stride)
    for b in range(batch):
        used = (kv_lens[b] + bs - 1) // bs
        table[b, used:] = -1
        if used > 1 and rng.random() < 0.5:
            table[b, rng.integers(0, used - 1)] = -1  # a hole in the cached prefix
    total = int(q_lens.sum())
    q = oracle.bf16_bits(rng.standard_normal((total, qh, 128)).astype(np.float32))
    k = oracle.bf16_bits(rng.standard_normal(blocks * bs * kvh * 128).astype(np.float32))
    v = oracle.bf16_bits(rng.standard_normal(blocks * bs * kvh * 128).astype(np.float32))
    cu = np.concatenate([[0], np.cumsum(q_lens)]).astype(np.int32)
    out, lse = oracle.attention_varlen(q, k, v, cu, kv_lens, table.ravel(), qh=qh, kvh=kvh, bs=bs, blocks=blocks,
                                       stride=stride)
    qf = _from_bf16(q).reshape(total, qh, 128)
    kf = _from_bf16(k).reshape(blocks * bs, kvh, 128)
    vf = _from_bf16(v).reshape(blocks * bs, kvh, 128)
    for b in range(batch):
        keys = np.arange(kv_lens[b])
        pages = table[b, keys // bs]
        slots = pages * bs + keys % bs
        for i in range(q_lens[b]):
            row = cu[b] + i
            vis = (keys <= kv_lens[b] - q_lens[b] + i) & (pages >= 0)
            for h in range(qh):
                kh = h // (qh // kvh)
                if not vis.any():
                    assert np.all(out[row, h] == 0) and np.isneginf(lse[b, h, i])
                    continue
                s = kf[slots[vis], kh] @ qf[row, h] / math.sqrt(128)
                m = s.max()
                p = np.exp(s - m)
                ref = p @ vf[slots[vis], kh] / p.sum()
                assert np.abs(out[row, h] - ref).max() < 2e-5, (b, i, h)
                assert abs(lse[b, h, i] - (m + math.log(p.sum()))) < 1e-4, (b, i, h)


def _bf16_rne(x):
    # float32 -> bf16 bits, round to nearest even (finite inputs)
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


@pytest.mark.parametrize("seed", range(6))
def test_fused_rope_cached_matches_float32_numpy(oracle, seed):
    # The cached fused kernel's oracle against a float32 numpy restatement of
    # kernels/kernels.cu:166-211, bit for bit: sequential f32 sum of squares,
    # 1 / sqrt(sum / dim + eps), (x * inv_rms) * w rounded to BF16 (:185),
    # rotate-half with separately rounded products (:203-204), Q to qout, K
    # (rotated) and V (copied) to their slot, slots outside the cache skipped,
    # positions past the table rotated by cos 1 / sin 0.
    rng = np.random.default_rng(seed)
    kvh = int(rng.choice([1, 2, 4]))
    qh = kvh * int(rng.choice([1, 2, 4]))
    dim = int(rng.choice([64, 128]))
    bs, blocks, max_pos = 4, 6, 50
    rows = int(rng.integers(1, 12))
    half = dim // 2
    qkv_f = (rng.standard_normal((rows, qh + 2 * kvh, dim)) * rng.choice([0.05, 1.0, 8.0])).astype(np.float32)
    qkv = oracle.bf16_bits(qkv_f)
    qw = oracle.bf16_bits((1 + 0.02 * rng.standard_normal(dim)).astype(np.float32))
    kw = oracle.bf16_bits((1 + 0.02 * rng.standard_normal(dim)).astype(np.float32))
    positions = rng.integers(0, max_pos + 10, size=rows).astype(np.int32)
    slots = rng.permutation(bs * blocks + 4)[:rows].astype(np.int32) - 2  # some -2 / -1 / past the cache
    cache = oracle.rope_cache(max_pos, dim, 1e6)
    eps = np.float32(1e-6)
    qout = np.zeros((rows, qh, dim), np.uint16)
    kc = np.full(bs * blocks * kvh * dim, 0x1234, np.uint16)
    vc = kc.copy()
    oracle.qkv_rope(qkv, qw, kw, positions, slots, qout, kc, vc, qh=qh, kvh=kvh, dim=dim, bs=bs, blocks=blocks,
                    eps=float(eps), rope_cache=cache, max_positions=max_pos)

    x_all = oracle.bits_to_f32(qkv).reshape(rows, qh + 2 * kvh, dim).astype(np.float32)
    wq, wk = oracle.bits_to_f32(qw).astype(np.float32), oracle.bits_to_f32(kw).astype(np.float32)
    want_q = np.zeros_like(qout)
    want_k = np.full_like(kc, 0x1234).reshape(bs * blocks, kvh, dim)
    want_v = want_k.copy()
    for r in range(rows):
        p = int(positions[r])
        c = cache[p, :half] if p < max_pos else np.ones(half, np.float32)
        s = cache[p, half:] if p < max_pos else np.zeros(half, np.float32)
        c, s = np.concatenate([c, c]), np.concatenate([s, s])
        for head in range(qh + kvh):
            x = x_all[r, head]
            total = np.cumsum(x * x, dtype=np.float32)[-1]
            inv = np.float32(1) / np.sqrt(total / np.float32(dim) + eps)
            w = wq if head < qh else wk
            n = oracle.bits_to_f32(_bf16_rne((x * inv) * w)).astype(np.float32)
            partner = np.concatenate([n[half:], n[:half]])
            a, b = n * c, partner * s
            rot = np.concatenate([a[:half] - b[:half], a[half:] + b[half:]])
            if head < qh:
                want_q[r, head] = _bf16_rne(rot)
            elif 0 <= slots[r] < bs * blocks:
                want_k[slots[r], head - qh] = _bf16_rne(rot)
                want_v[slots[r], head - qh] = qkv.reshape(rows, qh + 2 * kvh, dim)[r, qh + kvh + head - qh]
    assert np.array_equal(qout, want_q)
    assert np.array_equal(kc.reshape(want_k.shape), want_k)
    assert np.array_equal(vc.reshape(want_v.shape), want_v)
