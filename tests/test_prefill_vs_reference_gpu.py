"""Varlen and chunked prefill against the reference's own native kernel.

The reference runs prefill through `nv_attention` (kernels/kernels.cu:288-354,
475-485) on flattened rows: row r of sequence b is query i of that sequence
at position prefix_b + i (prefix_b = kv_len_b - q_len_b), so it attends to
positions[r] + 1 keys of block-table row b. The same seeded inputs go through
this library's nvb_paged_fwd_ex (cu_q / kv_lens form, tcgen05 prefill
kernels) and through the reference kernel built from its sources
(oracle/_ref/libref_native.so). Both are BF16 outputs of FP32 softmax
arithmetic in different orders; the bound is the north-star tolerance,
max-abs 2e-2 / mean-abs 2e-3. The reference kernel caps the context at its
max_context (4096 here), so every case stays within it.
"""
import pytest
import torch

from conftest import as_f32, assert_close

pytestmark = pytest.mark.gpu

MAX_CONTEXT = 4096


def _native_rows(case):
    """positions / seq_indices of the flattened rows (bottom-right causal)."""
    cu = case.cu_q.tolist()
    lens = case.kv_lens.tolist()
    pos, seq = [], []
    for b in range(case.batch):
        n = cu[b + 1] - cu[b]
        start = lens[b] - n
        pos.extend(range(start, start + n))
        seq.extend([b] * n)
    dev = case.q.device
    return (torch.tensor(pos, dtype=torch.int32, device=dev), torch.tensor(seq, dtype=torch.int32, device=dev))


def _mine(nvb, case):
    out = torch.empty_like(case.q)
    nvb.paged_fwd(case.q, case.k, case.v, out, case.cu_q, case.kv_lens, case.block_table, batch=case.batch,
                  max_q=case.max_q, max_k=int(case.kv_lens.max()), q_heads=case.q_heads, kv_heads=case.kv_heads,
                  block_size=case.block_size, table_stride=case.table_stride, num_blocks=case.num_blocks)
    torch.cuda.synchronize()
    return out


def _reference(ref_native, case):
    positions, seqs = _native_rows(case)
    out = torch.empty_like(case.q)
    rows = case.q.shape[0]
    ref_native.call("nv_attention", case.q, case.k, case.v, positions, seqs, case.block_table, out, rows,
                    case.q_heads, case.kv_heads, 128, case.block_size, case.num_blocks, case.table_stride,
                    case.batch, MAX_CONTEXT)
    return out


def _compare(nvb, ref_native, case, what):
    assert int(case.kv_lens.max()) <= MAX_CONTEXT
    nvb.clear_device_error()
    mine = _mine(nvb, case)
    ref = _reference(ref_native, case)
    assert_close(as_f32(mine), as_f32(ref), 2e-2, 2e-3, f"{what}: nvb_paged_fwd_ex vs reference nv_attention")
    assert nvb.device_error() == 0


def test_config2_prompts_match_reference_native_kernel(nvb, ref_native):
    # 32 prompts, L ~ U[64, 2048], 16q/8kv, N(0,1) inputs.
    _compare(nvb, ref_native, nvb.workloads.config2_prefill(seed=0), "config 2 prompts")


def test_config2_chunk64_over_prefix_matches_reference_native_kernel(nvb, ref_native):
    # The config's second pass: one 64-token chunk over a cached prefix P ~ U[256, 2048].
    _compare(nvb, ref_native, nvb.workloads.config2_chunked(seed=0), "config 2 chunk 64")


@pytest.mark.parametrize("q_heads,kv_heads", [(8, 8), (16, 4), (16, 2)])
def test_gqa_groups_match_reference_native_kernel(nvb, ref_native, q_heads, kv_heads):
    # GQA groups 1, 4 and 8: prompts of mixed length (one query tile, several
    # tiles, a tile boundary) and a 100-token chunk over a prefix.
    W = nvb.workloads
    kv = [700, 129, 1500, 64, 2200, 257]
    q = [700, 129, 1500, 64, 100, 257]
    case = W.paged_case(kv, q, q_heads=q_heads, kv_heads=kv_heads, seed=40 + q_heads + kv_heads, scale=1.0)
    _compare(nvb, ref_native, case, f"GQA {q_heads}q/{kv_heads}kv")
