"""Seeded random shapes through decode and prefill, against the CPU oracle.

Each seed draws one case that mixes what the fixed cases vary one at a time:
batch size, context and query lengths, kv heads, GQA group, page size and
(decode) split count; the short-chunk sweep keeps every sequence's queries
within one 128-row tile. Same tolerances as the fixed cases: max-abs 2e-2 /
mean-abs 2e-3 on the output, 1e-3 / 1e-4 on the LSE.
"""
import numpy as np
import pytest

from test_decode_gpu import _check as decode_check
from test_prefill_gpu import _check as prefill_check

pytestmark = pytest.mark.gpu

ORACLE_OPS = 3e9  # multiply-adds the scalar oracle does per case, at most


@pytest.mark.parametrize("seed", range(16))
def test_decode_random_shape(nvb, oracle, seed):
    rng = np.random.default_rng(1000 + seed)
    kvh = int(rng.choice([1, 2, 4, 8]))
    group = int(rng.choice([1, 2, 3, 4, 5, 8, 16]))
    bs = int(rng.choice([256, 512]))
    batch = int(rng.integers(1, 25))
    ctx = rng.integers(1, 3001, size=batch)
    while ctx.sum() * kvh * group * 256 > ORACLE_OPS:
        ctx = np.maximum(1, ctx // 2)
    splits = int(rng.choice([1, 2, 3, 7, 16]))
    case = nvb.workloads.paged_case(ctx.tolist(), q_heads=kvh * group, kv_heads=kvh, block_size=bs, seed=seed)
    decode_check(nvb, oracle, case, splits,
                 what=f"seed {seed}: batch {batch}, {kvh * group}q/{kvh}kv, block {bs}, ctx {ctx.min()}-{ctx.max()}")


@pytest.mark.parametrize("seed", range(12))
def test_prefill_random_shape(nvb, oracle, seed):
    rng = np.random.default_rng(2000 + seed)
    kvh = int(rng.choice([1, 2, 4, 8]))
    group = int(rng.choice([1, 2, 3, 4, 8, 16]))
    bs = int(rng.choice([256, 512]))
    batch = int(rng.integers(1, 7))
    q_lens = rng.integers(1, 301, size=batch)
    prefix = rng.integers(0, 1501, size=batch)
    while (q_lens * (prefix + q_lens)).sum() * kvh * group * 256 > ORACLE_OPS:
        q_lens, prefix = np.maximum(1, q_lens // 2), prefix // 2
    case = nvb.workloads.paged_case((prefix + q_lens).tolist(), q_lens.tolist(), q_heads=kvh * group,
                                    kv_heads=kvh, block_size=bs, seed=seed, scale=1.0)
    prefill_check(nvb, oracle, case,
                  what=f"seed {seed}: batch {batch}, {kvh * group}q/{kvh}kv, block {bs}, q {q_lens.tolist()}")


@pytest.mark.parametrize("seed", range(10))
def test_short_chunk_random_shape(nvb, oracle, seed):
    # Every sequence's queries fit one 128-row tile (q_len <= 128 / group):
    # chunked prefill of short chunks over long cached prefixes.
    rng = np.random.default_rng(3000 + seed)
    kvh = int(rng.choice([1, 2, 4, 8]))
    group = int(rng.choice([1, 2, 3, 4, 8, 16]))
    bs = int(rng.choice([256, 512]))
    batch = int(rng.integers(1, 41))
    q_lens = rng.integers(1, 128 // group + 1, size=batch)
    prefix = rng.integers(0, 3001, size=batch)
    while (q_lens * (prefix + q_lens)).sum() * kvh * group * 256 > ORACLE_OPS:
        prefix = prefix // 2
    case = nvb.workloads.paged_case((prefix + q_lens).tolist(), q_lens.tolist(), q_heads=kvh * group,
                                    kv_heads=kvh, block_size=bs, seed=seed, scale=1.0)
    prefill_check(nvb, oracle, case,
                  what=f"seed {seed}: batch {batch}, {kvh * group}q/{kvh}kv, block {bs}, q <= {128 // group}")
