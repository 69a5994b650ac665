"""GQA groups above 16 query heads per kv head, as the reference accepts them
(kernels/flash_native/flash_native.cu:48-52: any q_heads <= 256 that is a
multiple of kv_heads; its native kernel runs one CTA per query head).

* Decode: the tensor-core decode runs 16-head groups per CTA (adjacent CTAs
  of one kv head), with and without split-KV, including a group that is not
  a multiple of 16.
* Prefill: the tcgen05 prefill kernels pack 128 / group queries of the group
  per 128-row tile up to group 128 (one query per tile); past that the
  CUDA-core per-row decode takes the shape.
* The native (positions / seq_indices) form against the reference's own
  nv_attention built from source.
Tolerances as the other attention tests: max-abs 2e-2 / mean-abs 2e-3 on the
output, 1e-3 / 1e-4 on the LSE, against the FP32 oracle.
"""
import pytest
import torch

from conftest import as_f32, assert_close
from test_decode_gpu import _check as decode_check
from test_decode_gpu import _native_inputs
from test_prefill_gpu import _check as prefill_check

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qh,kvh", [(32, 1), (64, 2), (40, 1), (256, 1)])
def test_decode_large_groups(nvb, oracle, qh, kvh):
    case = nvb.workloads.paged_case([33, 400, 1023, 1, 256, 257], q_heads=qh, kv_heads=kvh, seed=qh * 7 + kvh)
    for splits in (1, 3):
        decode_check(nvb, oracle, case, splits, what=f"{qh}q/{kvh}kv decode")


def test_decode_large_group_auto_splits(nvb, oracle):
    case = nvb.workloads.paged_case([3000, 2500], q_heads=64, kv_heads=2, seed=5)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    splits = nvb.num_splits(case.batch, case.q_heads, case.kv_heads, 3000, sms)
    assert 1 <= splits <= 128
    decode_check(nvb, oracle, case, splits, what="64q/2kv auto splits")


@pytest.mark.parametrize("qh,kvh", [(32, 1), (64, 2), (128, 1), (256, 1)])
def test_prefill_large_groups(nvb, oracle, qh, kvh):
    # q lens past and within one query tile (128 / group queries), over
    # cached prefixes, with a one-token query.
    q_lens = [37, 5, 1, 64]
    prefix = [300, 0, 700, 129]
    case = nvb.workloads.paged_case([p + q for p, q in zip(prefix, q_lens)], q_lens, q_heads=qh, kv_heads=kvh,
                                    seed=qh + 3 * kvh, scale=1.0)
    prefill_check(nvb, oracle, case, what=f"{qh}q/{kvh}kv prefill")


@pytest.mark.parametrize("qh,kvh", [(32, 1), (64, 2)])
def test_short_chunk_large_groups(nvb, oracle, qh, kvh):
    # Every sequence's queries within one tile: the one-tile prefill kernel.
    group = qh // kvh
    q_lens = [max(1, 128 // group), 1, 2]
    prefix = [1000, 256, 37]
    case = nvb.workloads.paged_case([p + q for p, q in zip(prefix, q_lens)], q_lens, q_heads=qh, kv_heads=kvh,
                                    seed=11 + qh, scale=1.0)
    prefill_check(nvb, oracle, case, what=f"{qh}q/{kvh}kv short chunks")


@pytest.mark.parametrize("qh,kvh", [(32, 1), (64, 2)])
def test_native_large_groups_match_reference_native_kernel(nvb, ref_native, qh, kvh):
    case = nvb.workloads.paged_case([700, 33, 1500, 256], q_heads=qh, kv_heads=kvh, seed=qh + kvh)
    positions, seqs = _native_inputs(case)
    b = case.batch
    mine = torch.empty_like(case.q)
    nvb.attention(case.q, case.k, case.v, positions, seqs, case.block_table, mine, rows=b, q_heads=qh, kv_heads=kvh,
                  head_dim=128, block_size=256, num_blocks=case.num_blocks, table_stride=case.table_stride, batch=b,
                  max_context=4096)
    torch.cuda.synchronize()
    ref = torch.empty_like(case.q)
    ref_native.call("nv_attention", case.q, case.k, case.v, positions, seqs, case.block_table, ref, b, qh, kvh, 128,
                    256, case.num_blocks, case.table_stride, b, 4096)
    assert_close(as_f32(mine), as_f32(ref), 2e-2, 2e-3, f"{qh}q/{kvh}kv vs reference nv_attention")
