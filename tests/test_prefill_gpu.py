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


@pytest.mark.parametrize("qh,kvh", [(8, 8), (32, 8), (64, 8), (40, 8)])
def test_prefill_group_sizes(nvb, oracle, qh, kvh):
    W = nvb.workloads
    case = W.paged_case([129, 300, 520], [129, 45, 260], q_heads=qh, kv_heads=kvh, seed=qh, scale=1.0)
    _check(nvb, oracle, case, what=f"{qh}q/{kvh}kv")


def test_single_query_rows_mixed_with_long_groups(nvb, oracle):
    W = nvb.workloads
    case = W.paged_case([1, 513, 2, 700], [1, 300, 2, 1], q_heads=16, kv_heads=8, seed=21, scale=1.0)
    _check(nvb, oracle, case, what="mixed q lens")
