"""The allocation-free split-KV decode entry point, called through the C ABI.

Callers that cannot allocate device memory (a plugin inside a process that
owns the CUDA allocator, a fixed memory budget) use
nvb_paged_decode_static_scratch, whose split partials live in the library's
own fixed device array. Its output must match the regular entry point
(nvb_paged_fwd_ex with caller-owned scratch) within the tolerance of the
decode tests, on two calls in a row (the second call reuses the array the
first one left behind). This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

from conftest import as_f32, assert_close

pytestmark = pytest.mark.gpu

P, I = ctypes.c_void_p, ctypes.c_int


def _entry(nvb):
    fn = nvb.library().nvb_paged_decode_static_scratch
    fn.argtypes = [P] * 8 + [I] * 7 + [P, I]
    fn.restype = I
    return fn


def _ptr(t):
    return P(t.data_ptr()) if t is not None else P(0)


def _regular(nvb, case, splits):
    b, qh = case.batch, case.q_heads
    out = torch.empty_like(case.q)
    lse = torch.empty(b, qh, 1, dtype=torch.float32, device="cuda")
    la, oa = nvb.splitkv_scratch(splits, b, qh, "cuda")
    nvb.paged_fwd(case.q, case.k, case.v, out, case.cu_q, case.kv_lens, case.block_table, batch=b, max_q=1,
                  max_k=case.table_stride * case.block_size, q_heads=qh, kv_heads=case.kv_heads,
                  block_size=case.block_size, table_stride=case.table_stride, num_blocks=case.num_blocks,
                  num_splits=splits, lse=lse, lse_accum=la, out_accum=oa)
    return out, lse


def _static(nvb, case, splits):
    b, qh = case.batch, case.q_heads
    out = torch.empty_like(case.q)
    lse = torch.empty(b, qh, 1, dtype=torch.float32, device="cuda")
    stream = P(torch.cuda.current_stream().cuda_stream)
    rc = _entry(nvb)(stream, _ptr(case.q), _ptr(case.k), _ptr(case.v), _ptr(out), _ptr(case.cu_q),
                     _ptr(case.kv_lens), _ptr(case.block_table), b, case.table_stride * case.block_size, qh,
                     case.kv_heads, case.block_size, case.table_stride, splits, _ptr(lse), case.num_blocks)
    assert rc == 0, nvb.library().nvb_last_error()
    return out, lse


def test_static_scratch_matches_regular_entry_two_calls_in_a_row(nvb):
    W = nvb.workloads
    first = W.config1_decode(seed=0)                                   # 16q/8kv, ctx U[128, 1024]
    second = W.paged_case([4000, 37, 900, 1, 2049], q_heads=32, kv_heads=8, seed=5)
    for case, splits in ((first, 8), (second, 16)):
        got, got_lse = _static(nvb, case, splits)
        want, want_lse = _regular(nvb, case, splits)
        torch.cuda.synchronize()
        assert_close(as_f32(got), as_f32(want), 2e-2, 2e-3, f"static vs regular (splits={splits})")
        assert_close(got_lse.cpu().numpy(), want_lse.cpu().numpy(), 1e-3, 1e-4, "lse")
    assert nvb.device_error() == 0


def test_static_scratch_at_exactly_its_capacity(nvb):
    # 16 splits x 32 sequences x 32 heads = 16384 partials: the whole array,
    # including the last partials and the LSE block behind them, is used.
    case = nvb.workloads.paged_case([4096] * 31 + [300], q_heads=32, kv_heads=8, seed=9)
    nvb.clear_device_error()
    for _ in range(2):
        got, got_lse = _static(nvb, case, 16)
        want, want_lse = _regular(nvb, case, 16)
        torch.cuda.synchronize()
        assert_close(as_f32(got), as_f32(want), 2e-2, 2e-3, "static vs regular at 16384 partials")
        assert_close(got_lse.cpu().numpy(), want_lse.cpu().numpy(), 1e-3, 1e-4, "lse at 16384 partials")
    assert nvb.device_error() == 0


def test_static_scratch_rejects_calls_beyond_its_capacity(nvb):
    case = nvb.workloads.paged_case([300] * 8, q_heads=32, kv_heads=8, seed=1)
    out = torch.empty_like(case.q)
    stream = P(torch.cuda.current_stream().cuda_stream)
    # 128 splits x 8 sequences x 32 heads = 32768 partials > 16384
    rc = _entry(nvb)(stream, _ptr(case.q), _ptr(case.k), _ptr(case.v), _ptr(out), _ptr(case.cu_q),
                     _ptr(case.kv_lens), _ptr(case.block_table), 8, 512, 32, 8, 256, case.table_stride, 128, P(0),
                     case.num_blocks)
    assert rc == -1
    assert b"at most 16384" in nvb.library().nvb_last_error()
