"""Native-form attention for head sizes other than 128 (csrc/generic.cu), the
reference's head_dim dispatch and generic kernel (kernels/kernels.cu:226-271,
475-485).

Against the FP32 oracle for 40, 64, 96 and 256, and against the reference's
own native kernel for the sizes it instantiates (64, 256). Tolerance as the
decode tests: max-abs 2e-2 / mean-abs 2e-3. Rows with invalid sequences or
contexts must come out as zeros, and an invalid page masks its tokens.
"""
import pytest
import torch

from conftest import as_f32, assert_close, bits

pytestmark = pytest.mark.gpu


def _case(nvb, dim, lens, qh, kvh, seed, bs=256):
    base = nvb.workloads.paged_case(lens, q_heads=qh, kv_heads=kvh, block_size=bs, seed=seed)
    g = torch.Generator(device="cuda").manual_seed(1000 + seed)
    rows = len(lens)
    q = (torch.randn(rows, qh, dim, generator=g, device="cuda") * 0.5).bfloat16()
    k = (torch.randn(base.num_blocks, bs, kvh, dim, generator=g, device="cuda") * 0.5).bfloat16()
    v = (torch.randn(base.num_blocks, bs, kvh, dim, generator=g, device="cuda") * 0.5).bfloat16()
    positions = (base.kv_lens - 1).to(torch.int32)
    seqs = torch.arange(rows, dtype=torch.int32, device="cuda")
    return base, q, k, v, positions, seqs


def _mine(nvb, base, q, k, v, positions, seqs, dim, qh, kvh, max_context=1 << 20):
    out = torch.full_like(q, 7.0)
    nvb.attention(q, k, v, positions, seqs, base.block_table, out, rows=q.shape[0], q_heads=qh, kv_heads=kvh,
                  head_dim=dim, block_size=base.block_size, num_blocks=base.num_blocks, table_stride=base.table_stride,
                  batch=base.batch, max_context=max_context)
    torch.cuda.synchronize()
    return out


def _oracle(oracle, base, q, k, v, positions, seqs, dim, qh, kvh, max_context=1 << 20):
    return oracle.attention_native(bits(q), bits(k), bits(v), positions.cpu().numpy(), seqs.cpu().numpy(),
                                   base.block_table.cpu().numpy(), qh=qh, kvh=kvh, dim=dim, bs=base.block_size,
                                   blocks=base.num_blocks, stride=base.table_stride, batch=base.batch,
                                   max_context=max_context, threads=8)


@pytest.mark.parametrize("dim,qh,kvh", [(40, 8, 2), (64, 16, 8), (96, 12, 4), (256, 8, 8)])
def test_generic_head_dim_matches_oracle(nvb, oracle, dim, qh, kvh):
    base, q, k, v, pos, seqs = _case(nvb, dim, [700, 33, 1500], qh, kvh, seed=dim)
    out = _mine(nvb, base, q, k, v, pos, seqs, dim, qh, kvh)
    ref = _oracle(oracle, base, q, k, v, pos, seqs, dim, qh, kvh)
    assert_close(as_f32(out), ref, 2e-2, 2e-3, what=f"head_dim {dim}")


@pytest.mark.parametrize("dim", [64, 256])
def test_generic_head_dim_matches_reference_kernel(nvb, ref_native, dim):
    qh, kvh = 16, 8
    base, q, k, v, pos, seqs = _case(nvb, dim, [512, 1000, 77, 2048], qh, kvh, seed=dim + 1)
    out = _mine(nvb, base, q, k, v, pos, seqs, dim, qh, kvh, max_context=4096)
    ref = torch.empty_like(q)
    ref_native.call("nv_attention", q, k, v, pos, seqs, base.block_table, ref, q.shape[0], qh, kvh, dim,
                    base.block_size, base.num_blocks, base.table_stride, base.batch, 4096)
    assert_close(as_f32(out), as_f32(ref), 2e-2, 2e-3, what=f"head_dim {dim} vs reference nv_attention")


def test_generic_invalid_rows_and_pages(nvb, oracle):
    dim, qh, kvh = 64, 4, 2
    base, q, k, v, pos, seqs = _case(nvb, dim, [600, 300], qh, kvh, seed=5)
    base.block_table[0, 1] = -1  # tokens 256..511 of sequence 0 are masked
    seqs[1] = 9                  # row 1 names a sequence outside the batch
    out = _mine(nvb, base, q, k, v, pos, seqs, dim, qh, kvh)
    assert torch.all(out[1] == 0)
    ref = _oracle(oracle, base, q, k, v, pos, seqs, dim, qh, kvh)
    assert_close(as_f32(out[:1]), ref[:1], 2e-2, 2e-3, what="invalid page")


def test_generic_rejects_unsupported(nvb):
    base, q, k, v, pos, seqs = _case(nvb, 64, [100], 4, 2, seed=6)
    out = torch.empty_like(q)
    scratch = torch.empty(1 * 4 * 2 * (64 + 2), dtype=torch.float32, device="cuda")
    with pytest.raises(nvb.NvbError):  # split partitions exist for head_dim 128 only
        nvb.attention(q, k, v, pos, seqs, base.block_table, out, rows=1, q_heads=4, kv_heads=2, head_dim=64,
                      block_size=256, num_blocks=base.num_blocks, table_stride=base.table_stride, batch=1,
                      max_context=4096, scratch=scratch, partitions=2)
