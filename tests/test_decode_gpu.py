"""Split-KV paged decode attention on the GPU against the CPU oracle and the
reference's own native kernel.

Tolerance (BF16 output vs the FP32 oracle): max-abs 2e-2 and mean-abs 2e-3
for the random N(0,1)*0.5 benchmark inputs; the reference's own smoke cases
keep their bound of 3e-3 (kernels/flash_native/smoke.cu:84) and the ragged
GQA case its 4e-3 (src/gpu.rs:1459).
"""
import math

import numpy as np
import pytest
import torch

from conftest import as_f32, assert_close, bits

pytestmark = pytest.mark.gpu

TOL_MAX, TOL_MEAN = 2e-2, 2e-3


def _run(nvb, case, splits, max_k=None, stream=None):
    b, qh = case.batch, case.q_heads
    out = torch.empty_like(case.q)
    lse = torch.full((b, qh, 1), float("nan"), dtype=torch.float32, device="cuda")
    la, oa = (nvb.splitkv_scratch(splits, b, qh, "cuda") if splits > 1 else (None, None))
    nvb.paged_fwd(case.q, case.k, case.v, out, case.cu_q, case.kv_lens, case.block_table, batch=b, max_q=1,
                  max_k=max_k or case.table_stride * case.block_size, q_heads=qh, kv_heads=case.kv_heads,
                  block_size=case.block_size, table_stride=case.table_stride, num_blocks=case.num_blocks,
                  num_splits=splits, lse=lse, lse_accum=la, out_accum=oa, stream=stream)
    torch.cuda.synchronize()
    return out, lse


def _oracle(oracle, case, threads=8):
    return oracle.attention_varlen(bits(case.q), bits(case.k), bits(case.v), case.cu_q.cpu().numpy(),
                                   case.kv_lens.cpu().numpy(), case.block_table.cpu().numpy(), qh=case.q_heads,
                                   kvh=case.kv_heads, bs=case.block_size, blocks=case.num_blocks,
                                   stride=case.table_stride, threads=threads)


def _check(nvb, oracle, case, splits, tol=(TOL_MAX, TOL_MEAN), what=""):
    out, lse = _run(nvb, case, splits)
    ref, ref_lse = _oracle(oracle, case)
    assert_close(as_f32(out), ref, *tol, what=f"{what} out (splits={splits})")
    assert_close(lse.cpu().numpy(), ref_lse, 1e-3, 1e-4, what=f"{what} lse (splits={splits})")


@pytest.mark.parametrize("splits", [1, 2, 5, 8, 32])
def test_config1_decode_vs_oracle(nvb, oracle, splits):
    case = nvb.workloads.config1_decode()
    _check(nvb, oracle, case, splits, what="config1")


@pytest.mark.parametrize("splits", [1, 3])
def test_decode_block_size_512(nvb, oracle, splits):
    # 512-token pages: four 128-token tiles per page in the tensor-core decode,
    # with and without split-KV.
    case = nvb.workloads.paged_case([1500, 513, 2048, 90], q_heads=32, kv_heads=8, block_size=512, seed=19)
    _check(nvb, oracle, case, splits, what="block 512")


def test_config1_auto_splits(nvb, oracle):
    case = nvb.workloads.config1_decode()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    splits = nvb.num_splits(case.batch, case.q_heads, case.kv_heads, 4096, sms)
    assert 1 <= splits <= 128
    _check(nvb, oracle, case, splits, what="config1 auto")


@pytest.mark.parametrize("qh,kvh", [(8, 8), (16, 8), (32, 8), (40, 8), (64, 8), (16, 1), (48, 4)])
def test_gqa_group_sizes(nvb, oracle, qh, kvh):
    case = nvb.workloads.paged_case([33, 400, 1023, 1, 256, 257], q_heads=qh, kv_heads=kvh, seed=qh + kvh)
    for splits in (1, 3):
        _check(nvb, oracle, case, splits, what=f"{qh}q/{kvh}kv")


def _smoke_case(nvb, klens, h=16, hk=8):
    """Deterministic inputs of kernels/flash_native/smoke.cu:20-37."""
    d, page, stride, pages = 128, 256, 4, 12
    table = torch.tensor([7, 2, 10, 1, 3, 8, 0, 6, 11, 5, 9, 4], dtype=torch.int32).view(3, stride)
    nq = len(klens)
    iq = torch.arange(nq * h * d, dtype=torch.float64)
    ik = torch.arange(pages * page * hk * d, dtype=torch.float64)
    q = (torch.sin((iq % 1103) * 0.27) * 0.4).float().bfloat16().view(nq, h, d)
    k = (torch.cos((ik % 1091) * 0.19) * 0.3).float().bfloat16().view(pages, page, hk, d)
    v = (torch.sin((ik % 907) * 0.07) * 0.6).float().bfloat16().view(pages, page, hk, d)
    W = nvb.workloads
    return W.PagedCase(q=q.cuda(), k=k.cuda(), v=v.cuda(), block_table=table[:nq].contiguous().cuda(),
                       kv_lens=torch.tensor(klens, dtype=torch.int32, device="cuda"),
                       cu_q=torch.arange(nq + 1, dtype=torch.int32, device="cuda"), q_heads=h, kv_heads=hk,
                       block_size=page, table_stride=stride, num_blocks=pages)


@pytest.mark.parametrize("splits", [1, 2, 8, 32])
def test_reference_smoke_gqa_decode(nvb, oracle, splits):
    # kernels/flash_native/smoke.cu:89 (paged_gqa_decode), bound 3e-3.
    _check(nvb, oracle, _smoke_case(nvb, [33, 400, 1023]), splits, tol=(3e-3, 3e-3), what="smoke gqa")


@pytest.mark.parametrize("h,hk", [(8, 8), (16, 1)])
def test_reference_smoke_mha_mqa_decode(nvb, oracle, h, hk):
    # kernels/flash_native/smoke.cu:90-91 (paged_mha_decode, paged_mqa_decode).
    _check(nvb, oracle, _smoke_case(nvb, [33, 400, 1023], h, hk), 8, tol=(3e-3, 3e-3), what=f"smoke {h}/{hk}")


def test_graph_replay_after_changing_kv_lens(nvb, oracle):
    # kernels/flash_native/smoke.cu:45-53: capture, change device kv_lens, replay.
    case = _smoke_case(nvb, [33, 400, 1023])
    b, qh, splits = case.batch, case.q_heads, 8
    out = torch.empty_like(case.q)
    lse = torch.empty(b, qh, 1, dtype=torch.float32, device="cuda")
    la, oa = nvb.splitkv_scratch(splits, b, qh, "cuda")
    stream = torch.cuda.Stream()
    kw = dict(batch=b, max_q=1, max_k=1024, q_heads=qh, kv_heads=case.kv_heads, block_size=256,
              table_stride=case.table_stride, num_blocks=case.num_blocks, num_splits=splits, lse=lse,
              lse_accum=la, out_accum=oa, stream=stream)

    def step():
        nvb.paged_fwd(case.q, case.k, case.v, out, case.cu_q, case.kv_lens, case.block_table, **kw)

    with torch.cuda.stream(stream):
        step()  # warm-up outside capture encodes the TMA descriptors
    stream.synchronize()
    graph = nvb.capture(step, keep=[case, out, lse, la, oa], stream=stream)
    case.kv_lens.copy_(torch.tensor([40, 450, 700], dtype=torch.int32))
    torch.cuda.synchronize()
    graph.replay(stream)
    stream.synchronize()
    ref, _ = _oracle(oracle, case)
    assert_close(as_f32(out), ref, 3e-3, 3e-3, "graph replay")
    graph.close()


def test_known_answer_uniform_softmax_reversed_pages(nvb):
    # src/gpu.rs:1330-1358 at head_dim 128 / block_size 256: q = 0 gives a
    # uniform softmax, logical token t of value 1 + t over reversed physical
    # pages, so row r (context r + 1) averages to 1 + r / 2 exactly.
    rows, qh, kvh, bs = 3, 2, 1, 256
    q = torch.zeros(rows, qh, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(2, bs, kvh, 128, dtype=torch.bfloat16, device="cuda")
    v = torch.zeros_like(k)
    # tables [1, 0]: logical page 0 is physical page 1
    for t in range(3):
        v[1, t] = 1.0 + t
    table = torch.tensor([[1, 0]], dtype=torch.int32, device="cuda")
    positions = torch.tensor([0, 1, 2], dtype=torch.int32, device="cuda")
    seqs = torch.zeros(3, dtype=torch.int32, device="cuda")
    out = torch.full_like(q, 7.0)
    nvb.attention(q, k, v, positions, seqs, table, out, rows=rows, q_heads=qh, kv_heads=kvh, head_dim=128,
                  block_size=bs, num_blocks=2, table_stride=2, batch=1, max_context=512)
    torch.cuda.synchronize()
    got = as_f32(out)
    for r in range(rows):
        assert np.all(got[r] == 1.0 + 0.5 * r), (r, np.unique(got[r]))


def test_reference_ragged_gqa_case(nvb, oracle):
    # src/gpu.rs:1381-1471, the head_dim 128 / block_size 256 case, bound 4e-3.
    dim, bs, pos, seq, table = 128, 256, [0, 255, 256, 510], [0, 0, 1, 1], [3, 1, 0, 2]
    rows, qh, kvh, blocks = 4, 4, 2, 4
    iq = torch.arange(rows * qh * dim)
    ik = torch.arange(blocks * bs * kvh * dim)
    q = ((iq * 7 % 19).float() - 9) * 0.125
    k = ((ik * 11 % 23).float() - 11) * 0.125
    v = ((ik * 3 % 13).float() - 6) * 0.125
    qd = q.bfloat16().view(rows, qh, dim).cuda()
    kd = k.bfloat16().view(blocks, bs, kvh, dim).cuda()
    vd = v.bfloat16().view(blocks, bs, kvh, dim).cuda()
    p = torch.tensor(pos, dtype=torch.int32, device="cuda")
    s = torch.tensor(seq, dtype=torch.int32, device="cuda")
    t = torch.tensor(table, dtype=torch.int32, device="cuda").view(2, 2)
    out = torch.empty_like(qd)
    nvb.attention(qd, kd, vd, p, s, t, out, rows=rows, q_heads=qh, kv_heads=kvh, head_dim=dim, block_size=bs,
                  num_blocks=blocks, table_stride=2, batch=2, max_context=511)
    torch.cuda.synchronize()
    ref = oracle.attention_native(bits(qd), bits(kd), bits(vd), pos, seq, table, qh=qh, kvh=kvh, dim=dim, bs=bs,
                                  blocks=blocks, stride=2, batch=2, max_context=511)
    assert_close(as_f32(out), ref, 4e-3, 4e-3, "ragged gqa")


def _native_inputs(case):
    b = case.batch
    positions = (case.kv_lens - 1).to(torch.int32)
    seqs = torch.arange(b, dtype=torch.int32, device="cuda")
    return positions, seqs


def test_native_form_matches_reference_native_kernel(nvb, ref_native):
    case = nvb.workloads.config1_decode()
    positions, seqs = _native_inputs(case)
    b, qh, kvh = case.batch, case.q_heads, case.kv_heads
    mine = torch.empty_like(case.q)
    nvb.attention(case.q, case.k, case.v, positions, seqs, case.block_table, mine, rows=b, q_heads=qh, kv_heads=kvh,
                  head_dim=128, block_size=256, num_blocks=case.num_blocks, table_stride=case.table_stride, batch=b,
                  max_context=4096)
    torch.cuda.synchronize()
    ref = torch.empty_like(case.q)
    ref_native.call("nv_attention", case.q, case.k, case.v, positions, seqs, case.block_table, ref, b, qh, kvh, 128,
                    256, case.num_blocks, case.table_stride, b, 4096)
    # Both are BF16 outputs of FP32 math in different orders.
    assert_close(as_f32(mine), as_f32(ref), 2e-2, 2e-3, "vs reference nv_attention")


def test_native_splitkv_matches_reference_candidate(nvb, ref_native, oracle):
    case = nvb.workloads.config1_decode(seed=3)
    positions, seqs = _native_inputs(case)
    b, qh, kvh, parts = case.batch, case.q_heads, case.kv_heads, 16
    scratch = torch.empty(b * qh * parts * 130, dtype=torch.float32, device="cuda")
    mine = torch.empty_like(case.q)
    nvb.attention(case.q, case.k, case.v, positions, seqs, case.block_table, mine, rows=b, q_heads=qh, kv_heads=kvh,
                  head_dim=128, block_size=256, num_blocks=case.num_blocks, table_stride=case.table_stride, batch=b,
                  max_context=4096, scratch=scratch, partitions=parts)
    torch.cuda.synchronize()
    ref = torch.empty_like(case.q)
    ref_scratch = torch.empty_like(scratch)
    ref_native.call("nv_attention_splitkv_candidate", case.q, case.k, case.v, positions, seqs, case.block_table, ref,
                    b, qh, kvh, 128, 256, case.num_blocks, case.table_stride, b, 4096, ref_scratch, parts)
    assert_close(as_f32(mine), as_f32(ref), 2e-2, 2e-3, "vs reference split-KV candidate")
    expect, _ = _oracle(oracle, case)
    assert_close(as_f32(mine), expect, TOL_MAX, TOL_MEAN, "native split-KV vs oracle")


def test_native_invalid_rows_are_zero(nvb):
    case = nvb.workloads.paged_case([300, 40], q_heads=4, kv_heads=2, seed=9)
    b = case.batch
    positions = torch.tensor([299, 39], dtype=torch.int32, device="cuda")
    for bad_seq, bad_pos, maxc in ((5, 39, 4096), (1, -3, 4096), (1, 39, 10)):
        seqs = torch.tensor([0, bad_seq], dtype=torch.int32, device="cuda")
        pos = positions.clone()
        pos[1] = bad_pos
        out = torch.full_like(case.q, 3.0)
        nvb.attention(case.q, case.k, case.v, pos, seqs, case.block_table, out, rows=b, q_heads=4, kv_heads=2,
                      head_dim=128, block_size=256, num_blocks=case.num_blocks, table_stride=case.table_stride,
                      batch=b, max_context=maxc)
        torch.cuda.synchronize()
        assert torch.all(out[1] == 0), (bad_seq, bad_pos, maxc)
        if maxc > 300:  # row 0 (context 300) stays valid
            assert torch.all(torch.isfinite(out[0].float())) and not torch.all(out[0] == 0)


def test_invalid_page_masks_its_tokens(nvb, oracle):
    case = nvb.workloads.paged_case([700, 900], q_heads=8, kv_heads=2, seed=4)
    case.block_table[1, 1] = -1  # tokens 256..511 of sequence 1 are masked
    for splits in (1, 4):
        _check(nvb, oracle, case, splits, what="invalid page")


def test_context_edges(nvb, oracle):
    lens = [1, 2, 31, 32, 33, 255, 256, 257, 511, 512, 513]
    case = nvb.workloads.paged_case(lens, q_heads=16, kv_heads=8, seed=12)
    for splits in (1, 2, 7):
        _check(nvb, oracle, case, splits, what="context edges")


def test_long_context_config5_shard(nvb, oracle):
    # One GPU's shard of config 5: a kv head with its 8 query heads, ctx 32768.
    case = nvb.workloads.config5_decode(kv_heads=1, q_heads=8)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    splits = nvb.num_splits(case.batch, 8, 1, 32768, sms)
    _check(nvb, oracle, case, splits, what="ctx 32768")


@pytest.mark.parametrize("splits", [1, 7, 37, 74, 128])
def test_shard_split_counts(nvb, oracle, splits):
    # The config-5 shard of 8 GPUs in miniature: 4 ragged sequences x 1 kv head
    # (8 query heads), ctx up to 8192, split 1 to 128 ways (the combine with 1,
    # 2, 4 and 8 warps per item; 128 splits leave the short sequence's
    # trailing splits without keys).
    case = nvb.workloads.paged_case([8192, 8000, 7777, 129], q_heads=8, kv_heads=1, seed=31 + splits)
    _check(nvb, oracle, case, splits, what=f"{splits} splits")


def test_config3_full_size_sampled(nvb, oracle):
    # Full config 3 on the GPU; a sample of its sequences checked on the CPU.
    case = nvb.workloads.config3_decode()
    out, _ = _run(nvb, case, 1)
    sample = [0, 77, 128, 255]
    W = nvb.workloads
    sub = W.PagedCase(q=case.q[sample], k=case.k, v=case.v, block_table=case.block_table[sample].contiguous(),
                      kv_lens=case.kv_lens[sample].contiguous(),
                      cu_q=torch.arange(len(sample) + 1, dtype=torch.int32, device="cuda"), q_heads=32, kv_heads=8,
                      block_size=256, table_stride=case.table_stride, num_blocks=case.num_blocks)
    ref, _ = _oracle(oracle, sub)
    assert_close(as_f32(out[sample]), ref, TOL_MAX, TOL_MEAN, "config3 sample")
    assert nvb.device_error() == 0


def test_rejects_invalid_arguments(nvb):
    case = nvb.workloads.paged_case([10], q_heads=4, kv_heads=2, seed=1)
    out = torch.empty_like(case.q)
    base = dict(batch=1, max_q=1, max_k=256, q_heads=4, kv_heads=2, block_size=256, table_stride=1, num_blocks=1)
    for bad in (dict(block_size=128), dict(q_heads=5), dict(num_splits=129), dict(max_k=257)):
        kw = {**base, **bad}
        with pytest.raises(nvb.NvbError):
            nvb.paged_fwd(case.q, case.k, case.v, out, case.cu_q, case.kv_lens, case.block_table, check=False, **kw)
