"""Varlen and chunked causal prefill over the paged cache (max_q > 1).

Parity with the FP32 oracle of kernels/flash_native/smoke.cu:57-81 (queries
are the bottom-right suffix of each sequence's keys), max-abs 2e-2 /
mean-abs 2e-3 on N(0,1) inputs, 3e-3 on the reference's smoke inputs.
"""
import pytest
import torch

from conftest import as_f32, assert_close, bits

pytestmark = pytest.mark.gpu


def _run(nvb, case):
    b, qh = case.batch, case.q_heads
    out = torch.empty_like(case.q)
    lse = torch.full((b, qh, case.max_q), float("nan"), dtype=torch.float32, device="cuda")
    nvb.paged_fwd(case.q, case.k, case.v, out, case.cu_q, case.kv_lens, case.block_table, batch=b, max_q=case.max_q,
                  max_k=int(case.kv_lens.max()), q_heads=qh, kv_heads=case.kv_heads, block_size=case.block_size,
                  table_stride=case.table_stride, num_blocks=case.num_blocks, lse=lse)
    torch.cuda.synchronize()
    return out, lse


def _oracle(oracle, case):
    return oracle.attention_varlen(bits(case.q), bits(case.k), bits(case.v), case.cu_q.cpu().numpy(),
                                   case.kv_lens.cpu().numpy(), case.block_table.cpu().numpy(), qh=case.q_heads,
                                   kvh=case.kv_heads, bs=case.block_size, blocks=case.num_blocks,
                                   stride=case.table_stride, threads=8)


def _check(nvb, oracle, case, tol=(2e-2, 2e-3), what=""):
    out, lse = _run(nvb, case)
    ref, ref_lse = _oracle(oracle, case)
    assert_close(as_f32(out), ref, *tol, what=f"{what} out")
    # lse is padded to max_q per sequence; compare only real query slots.
    cu = case.cu_q.tolist()
    for b in range(case.batch):
        n = cu[b + 1] - cu[b]
        assert_close(lse[b, :, :n].cpu().numpy(), ref_lse[b, :, :n], 1e-3, 1e-4, what=f"{what} lse seq {b}")


def test_reference_smoke_ragged_prefill(nvb, oracle):
    # kernels/flash_native/smoke.cu:88: q lens {17, 65, 7}, kv lens {33, 400, 270}.
    from test_decode_gpu import _smoke_case

    case = _smoke_case(nvb, [33, 400, 270])
    # rebuild q for 17 + 65 + 7 query rows with the same formula
    qlens = [17, 65, 7]
    n = sum(qlens)
    iq = torch.arange(n * 16 * 128, dtype=torch.float64)
    case.q = (torch.sin((iq % 1103) * 0.27) * 0.4).float().bfloat16().view(n, 16, 128).cuda()
    cu = [0]
    for x in qlens:
        cu.append(cu[-1] + x)
    case.cu_q = torch.tensor(cu, dtype=torch.int32, device="cuda")
    _check(nvb, oracle, case, tol=(3e-3, 3e-3), what="smoke ragged prefill")


@pytest.mark.parametrize("seed", [0, 1])
def test_varlen_prefill_config2_shape(nvb, oracle, seed):
    W = nvb.workloads
    lens = W.uniform_lengths(6, 64, 700, seed)
    case = W.paged_case(lens, lens, q_heads=16, kv_heads=8, seed=seed, scale=1.0)
    _check(nvb, oracle, case, what="varlen prefill")


def test_chunked_prefill_over_cached_prefix(nvb, oracle):
    W = nvb.workloads
    prefix = [256, 300, 1000, 2047]
    case = W.paged_case([p + 64 for p in prefix], [64] * 4, q_heads=16, kv_heads=8, seed=7, scale=1.0)
    _check(nvb, oracle, case, what="chunk 64")


def test_chunked_prefill_pair_tiles_of_unequal_length(nvb, oracle):
    # 100-token chunks span two 64-query tiles (16q/8kv): the pair kernel. Over
    # a 960-token prefix tile A (queries 0-63) visits 8 KV tiles and tile B 9;
    # a 36-query chunk leaves tile B empty; a 2000-token prefix crosses pages.
    W = nvb.workloads
    prefix = [960, 1000, 40, 2000]
    q_lens = [100, 100, 36, 100]
    case = W.paged_case([p + q for p, q in zip(prefix, q_lens)], q_lens, q_heads=16, kv_heads=8, seed=8, scale=1.0)
    _check(nvb, oracle, case, what="chunk 100, unequal pair tiles")


@pytest.mark.parametrize("qh,kvh", [(8, 8), (32, 8), (64, 8), (40, 8)])
def test_prefill_group_sizes(nvb, oracle, qh, kvh):
    W = nvb.workloads
    case = W.paged_case([129, 300, 520], [129, 45, 260], q_heads=qh, kv_heads=kvh, seed=qh, scale=1.0)
    _check(nvb, oracle, case, what=f"{qh}q/{kvh}kv")


def test_single_query_rows_mixed_with_long_groups(nvb, oracle):
    W = nvb.workloads
    case = W.paged_case([1, 513, 2, 700], [1, 300, 2, 1], q_heads=16, kv_heads=8, seed=21, scale=1.0)
    _check(nvb, oracle, case, what="mixed q lens")


@pytest.mark.parametrize("qh,kvh", [(128, 8), (24, 8)])
def test_prefill_group_16_and_partial_rows(nvb, oracle, qh, kvh):
    # 16 heads per kv head (8 queries per 128-row sub-tile) and 3 heads per
    # kv head (126 of 128 rows used)
    W = nvb.workloads
    case = W.paged_case([77, 400, 1030], [77, 150, 300], q_heads=qh, kv_heads=kvh, seed=qh + 1, scale=1.0)
    _check(nvb, oracle, case, what=f"{qh}q/{kvh}kv")


def test_prefill_nan_past_kv_len_and_invalid_page(nvb, oracle):
    # Cache rows past each sequence's length hold NaN (they must meet only
    # P = 0 and be zeroed first); page 1 of sequence 1 is invalid (-1), so
    # keys 256..511 of that sequence are masked, as in the oracle.
    W = nvb.workloads
    case = W.paged_case([300, 700, 130], [300, 200, 130], q_heads=16, kv_heads=8, seed=5, scale=1.0)
    bs = case.block_size
    for b, n in enumerate(case.kv_lens.tolist()):
        page = int(case.block_table[b, (n - 1) // bs])
        if n % bs:
            case.k[page, n % bs:] = float("nan")
            case.v[page, n % bs:] = float("nan")
    case.block_table[1, 1] = -1
    out, _ = _run(nvb, case)
    assert torch.isfinite(out.float()).all()
    _check(nvb, oracle, case, what="nan tail / invalid page")


def test_prefill_more_items_than_sms(nvb, oracle):
    # 2500 + 1800 queries x 8 kv heads: more work items than SMs, so CTAs of
    # the persistent kernel run several items and reuse Q / O buffers.
    W = nvb.workloads
    case = W.paged_case([2500, 1800], [2500, 1800], q_heads=16, kv_heads=8, seed=11, scale=1.0)
    _check(nvb, oracle, case, what="persistent items")


@pytest.mark.parametrize("max_q", [130, 64])
def test_prefill_batch_beyond_ranking_limit(nvb, oracle, max_q):
    # More sequences than the kernels rank by work at start-up (1,024): items
    # are claimed in index order. Ragged queries over short cached prefixes
    # (16q/8kv, 64 queries per tile): up to 130 queries runs the pair kernel,
    # up to 64 the one-tile kernel.
    import numpy as np

    W = nvb.workloads
    rng = np.random.default_rng(12 + max_q)
    q_lens = rng.integers(1, max_q + 1, size=1100).tolist()
    q_lens[0] = max_q
    prefix = rng.integers(0, 201, size=1100).tolist()
    case = W.paged_case([p + q for p, q in zip(prefix, q_lens)], q_lens, q_heads=16, kv_heads=8, seed=13, scale=1.0)
    _check(nvb, oracle, case, what=f"1,100 sequences, up to {max_q} queries")


@pytest.mark.parametrize("q_lens", [[700, 200, 90], [64, 30, 64]])
def test_prefill_block_size_512(nvb, oracle, q_lens):
    # 512-token pages hold four 128-key tiles: the page of tile j is j / 4 and
    # its first row is offset within the page. [700, 200, 90] queries run the
    # pair kernel, [64, 30, 64] the one-tile kernel.
    W = nvb.workloads
    kv = [700, 1300, 1100]
    case = W.paged_case(kv, q_lens, q_heads=16, kv_heads=8, block_size=512, seed=17, scale=1.0)
    _check(nvb, oracle, case, what=f"block 512, q {q_lens}")


@pytest.mark.parametrize("q_len", [300, 64])
def test_prefill_concurrent_streams(nvb, q_len):
    # Two launches that overlap on the GPU, on two streams: each stream has its
    # own work-claim counters, so each result equals the same launch run
    # alone. 300-query prompts run the pair kernel, 64-query chunks the
    # one-tile kernel.
    W = nvb.workloads
    cases = [W.paged_case([q_len + p for p in prefix], [q_len] * 6, q_heads=16, kv_heads=8, seed=40 + i, scale=1.0)
             for i, prefix in enumerate(([0, 100, 900, 40, 2000, 300], [500, 0, 60, 1200, 7, 800]))]
    alone = [_run(nvb, c)[0] for c in cases]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [torch.empty_like(c.q) for c in cases]
    torch.cuda.synchronize()
    for rep in range(3):
        for c, o, st in zip(cases, outs, streams):
            with torch.cuda.stream(st):
                nvb.paged_fwd(c.q, c.k, c.v, o, c.cu_q, c.kv_lens, c.block_table, batch=c.batch, max_q=c.max_q,
                              max_k=int(c.kv_lens.max()), q_heads=16, kv_heads=8, block_size=c.block_size,
                              table_stride=c.table_stride, num_blocks=c.num_blocks, stream=st)
        torch.cuda.synchronize()
        assert nvb.device_error() == 0
        for o, a in zip(outs, alone):
            assert torch.equal(o, a), f"stream result differs from the lone launch (rep {rep})"


@pytest.mark.parametrize("q_len", [300, 64])
def test_prefill_chain_reads_previous_launch(nvb, q_len):
    # Each launch waits for the kernel before it on the stream before reading
    # any input (it starts early only to set up shared memory and TMEM). Here
    # every launch takes the previous launch's output as its queries, with no
    # host synchronisation in between: the results equal the same chain run
    # with a synchronise after each launch, bit for bit. 300-query prompts run
    # the pair kernel, 64-query chunks the one-tile kernel.
    W = nvb.workloads
    c = W.paged_case([q_len + p for p in (0, 700, 90, 1500)], [q_len] * 4, q_heads=16, kv_heads=8, seed=50, scale=1.0)
    kw = dict(batch=c.batch, max_q=c.max_q, max_k=int(c.kv_lens.max()), q_heads=16, kv_heads=8,
              block_size=c.block_size, table_stride=c.table_stride, num_blocks=c.num_blocks)

    def chain(sync):
        bufs = [c.q.clone()] + [torch.empty_like(c.q) for _ in range(4)]
        for i in range(4):
            nvb.paged_fwd(bufs[i], c.k, c.v, bufs[i + 1], c.cu_q, c.kv_lens, c.block_table, **kw)
            if sync:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        return bufs[1:]

    ref = chain(True)
    for rep in range(3):
        got = chain(False)
        assert nvb.device_error() == 0
        for i, (g, r) in enumerate(zip(got, ref)):
            assert torch.equal(g, r), f"launch {i} of the chain differs (rep {rep})"
