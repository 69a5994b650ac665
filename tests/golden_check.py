"""Inputs and checks for the golden fixtures in tests/golden/.

Inputs come from an exact integer hash (no RNG or libm dependence), so a
fixture stores only the reference kernels' outputs. make_golden.py writes the
fixtures by running the reference's own CUDA kernels (oracle/_ref) on a B200;
check() compares the CPU oracle against them.
"""
from __future__ import annotations

import numpy as np

QH, KVH, DIM, BS = 16, 8, 128, 256
EPS, THETA, MAXPOS = 1e-6, 1e6, 4096

# native attention case: row r attends to positions[r] + 1 keys of table row r
POSITIONS = np.array([32, 299, 700, 1023, 0, 255, 256], np.int32)
PAGES = [1, 2, 3, 4, 1, 1, 2]
NUM_BLOCKS = sum(PAGES) + 2
STRIDE = max(PAGES)
ROPE_ROWS = 9
ROPE_BLOCKS = 2
TABLE_ROWS_SAMPLED = np.array([0, 1, 2, 350, 4095], np.int32)


def hashed(n, salt, scale):
    """Deterministic values in [-scale, scale): a multiplicative hash of the index."""
    i = np.arange(n, dtype=np.uint64)
    h = (i * np.uint64(2654435761) + np.uint64(salt) * np.uint64(40503)) % np.uint64(1 << 32)
    h = (h ^ (h >> np.uint64(15))) * np.uint64(2246822519) % np.uint64(1 << 32)
    return ((h.astype(np.float64) / float(1 << 32)) * 2.0 - 1.0).astype(np.float32) * np.float32(scale)


def table():
    perm = [(7 * i + 3) % NUM_BLOCKS for i in range(NUM_BLOCKS)]
    t = np.full((len(PAGES), STRIDE), -1, np.int32)
    c = 0
    for r, n in enumerate(PAGES):
        t[r, :n] = perm[c:c + n]
        c += n
    return t


def attention_inputs(oracle):
    rows = len(POSITIONS)
    q = oracle.bf16_bits(hashed(rows * QH * DIM, 1, 1.5).reshape(rows, QH, DIM))
    k = oracle.bf16_bits(hashed(NUM_BLOCKS * BS * KVH * DIM, 2, 1.5).reshape(NUM_BLOCKS, BS, KVH, DIM))
    v = oracle.bf16_bits(hashed(NUM_BLOCKS * BS * KVH * DIM, 3, 1.5).reshape(NUM_BLOCKS, BS, KVH, DIM))
    return q, k, v, POSITIONS, np.arange(rows, dtype=np.int32), table()


def rope_inputs(oracle):
    qkv = oracle.bf16_bits(hashed(ROPE_ROWS * (QH + 2 * KVH) * DIM, 4, 3.0).reshape(ROPE_ROWS, QH + 2 * KVH, DIM))
    qw = oracle.bf16_bits(1.0 + hashed(DIM, 5, 0.05))
    kw = oracle.bf16_bits(1.0 + hashed(DIM, 6, 0.05))
    positions = np.array([0, 1, 350, 4095, 17, 2048, -3, 4100, 999], np.int32)
    slots = np.array([5, 0, 511, 300, -1, 12, 7, 8, 512], np.int32)  # -1 and 512 are skipped
    return qkv, qw, kw, positions, slots


def check(oracle, fx, name):
    if name.startswith("native_attention"):
        q, k, v, pos, seqs, tbl = attention_inputs(oracle)
        got = oracle.attention_native(q, k, v, pos, seqs, tbl.reshape(-1), qh=QH, kvh=KVH, dim=DIM, bs=BS,
                                      blocks=NUM_BLOCKS, stride=STRIDE, batch=len(PAGES), max_context=4096)
        for key in ("out", "splitkv_out"):
            ref = oracle.bits_to_f32(fx[key])
            err = np.abs(got - ref)
            # reference BF16 output vs FP32 oracle: one BF16 rounding plus
            # FP32 reordering
            assert err.max() <= 2e-2 and err.mean() <= 2e-3, (key, err.max(), err.mean())
    elif name.startswith("qkv_rope"):
        qkv, qw, kw, pos, slots = rope_inputs(oracle)
        table_rows = fx["rope_rows"]
        ref_table = oracle.rope_cache(MAXPOS, DIM, THETA)
        assert np.abs(ref_table[TABLE_ROWS_SAMPLED] - table_rows).max() <= 2e-3
        rope_table = np.zeros((MAXPOS, DIM), np.float32)
        rope_table[TABLE_ROWS_SAMPLED] = table_rows
        # use the reference's own table values for the sampled positions
        full = ref_table.copy()
        full[TABLE_ROWS_SAMPLED] = table_rows
        qout = np.zeros((ROPE_ROWS, QH, DIM), np.uint16)
        kc = np.zeros((ROPE_BLOCKS * BS * KVH * DIM,), np.uint16)
        vc = np.zeros_like(kc)
        oracle.qkv_rope(qkv, qw, kw, pos, slots, qout, kc, vc, qh=QH, kvh=KVH, dim=DIM, bs=BS, blocks=ROPE_BLOCKS,
                        eps=EPS, rope_cache=full, max_positions=MAXPOS)
        valid = (slots >= 0) & (slots < ROPE_BLOCKS * BS)
        idx = slots[valid]
        kc = kc.reshape(-1, KVH, DIM)[idx]
        vc = vc.reshape(-1, KVH, DIM)[idx]
        assert np.array_equal(vc, fx["v_slots"]), "V scatter differs from the reference kernel"
        for got, key in ((qout, "qout"), (kc, "k_slots")):
            a, b = oracle.bits_to_f32(got), oracle.bits_to_f32(fx[key])
            err = np.abs(a - b)
            # the CPU's 1/sqrtf vs the GPU's rsqrtf can move one BF16 rounding
            assert err.max() <= 0.0625 and (err > 0).mean() <= 0.02, (key, err.max(), (err > 0).mean())
    else:
        raise AssertionError(f"unknown fixture {name}")
