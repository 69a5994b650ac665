"""The decode-shaped tcgen05 GEMM (nvbe_layer_gemm) against an FP64 reference.

y = x w^T with BF16 inputs and output. Each output may differ from the exact
product by its own BF16 rounding (one unit in the last place of the larger
of the two magnitudes: a sum just below a power of two may round up into
the next binade) plus the error bound of an FP32 accumulation of K products,
K * 2^-24 * sum |x w| (what matters where the sum cancels towards zero, where
a BF16 ulp is smaller than any FP32 accumulation error). cuBLAS is held to
the same bound. The fused SiLU epilogue must equal the unfused GEMM followed
by the reference-identical SiLU kernel bit for bit (both sum each output in
the same order), and a second launch must reproduce the first bit for bit
(the cross-CTA split-K sum has a fixed order, so graph replays equal eager
runs).
"""
import pytest
import torch

import __graft_entry__
from conftest import bits

pytestmark = pytest.mark.gpu

M_ = __graft_entry__.load_package().model


def _operands(m, n, k, seed, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (torch.randn(m, k, generator=g, device="cuda") * scale).bfloat16()
    w = (torch.randn(n, k, generator=g, device="cuda") * 0.02).bfloat16()
    return x, w


def _ulp(v):
    a = v.abs().clamp_min(1e-30)
    return torch.exp2(torch.floor(torch.log2(a)) - 7)


def _reference(x, w):
    xd, wd = x.double(), w.double()
    return xd @ wd.t(), x.shape[1] * 2.0**-24 * (xd.abs() @ wd.abs().t())


def _assert_close(got, x, w, what, exact=None):
    ref, acc_bound = exact if exact is not None else _reference(x, w)
    g = got.double()
    diff = (g - ref).abs()
    allowed = _ulp(torch.maximum(ref.abs(), g.abs())) + acc_bound
    bad = diff > allowed
    assert not bad.any(), f"{what}: {int(bad.sum())} outputs beyond the bound, max diff {diff.max().item():.3e}"
    frac = (g != ref.float().bfloat16().double()).double().mean().item()
    assert frac < 0.02, f"{what}: {frac:.3%} of outputs differ from the rounded exact product"


@pytest.mark.parametrize("m,n,k", [(256, 4096, 1024), (256, 1024, 2048), (256, 1024, 3072), (1, 4096, 1024),
                                   (17, 1024, 2048), (100, 152, 64), (255, 2052, 192), (64, 2376, 1024)])
def test_gemm_matches_exact_reference(m, n, k):
    x, w = _operands(m, n, k, seed=m + n + k)
    y = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    M_.layer_gemm(x, w, y)
    torch.cuda.synchronize()
    assert M_.gemm_device_error() == 0
    _assert_close(y, x, w, f"{m}x{n}x{k}")


@pytest.mark.parametrize("m", [256, 33, 1])
def test_gemm_silu_fused_equals_unfused(m):
    inter, hidden = 3072, 1024
    x, w = _operands(m, 2 * inter, hidden, seed=7 + m, scale=3.0)
    packed = torch.empty(m, 2 * inter, dtype=torch.bfloat16, device="cuda")
    M_.layer_gemm(x, w, packed)
    unfused = torch.empty(m, inter, dtype=torch.bfloat16, device="cuda")
    M_.layer_silu_mul(packed, unfused)
    fused = torch.empty(m, inter, dtype=torch.bfloat16, device="cuda")
    M_.layer_gemm(x, w, fused, silu=True)
    torch.cuda.synchronize()
    assert M_.gemm_device_error() == 0
    assert (bits(fused) == bits(unfused)).all()
    _assert_close(packed, x, w, "gate/up")


def test_gemm_deterministic_and_within_cublas_bound():
    m, n, k = 256, 1024, 3072
    x, w = _operands(m, n, k, seed=3)
    a, b = (torch.empty(m, n, dtype=torch.bfloat16, device="cuda") for _ in range(2))
    M_.layer_gemm(x, w, a)
    M_.layer_gemm(x, w, b)
    torch.cuda.synchronize()
    assert (bits(a) == bits(b)).all()
    exact = _reference(x, w)
    _assert_close(a, x, w, "tcgen05 GEMM", exact)
    _assert_close(x @ w.t(), x, w, "cuBLAS (context)", exact)


def test_gemm_rejects_invalid_shapes():
    x, w = _operands(4, 128, 96, seed=1)  # K not a multiple of 64
    y = torch.empty(4, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(M_.ModelError):
        M_.layer_gemm(x, w, y)
    x, w = _operands(257, 128, 64, seed=1)  # more rows than the decode GEMM takes
    y = torch.empty(257, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(M_.ModelError):
        M_.layer_gemm(x, w, y)


@pytest.mark.parametrize("m,n", [(8, 151936), (16, 20000), (1, 151936), (37, 20000)])
def test_gemm_sample_fused_equals_unfused(m, n):
    """The LM head with the Gumbel-max sampler fused into its epilogue gives
    the same BF16 logits as the plain GEMM (both sum each logit in the same
    order: more 128-token tiles than SMs, so neither splits K) and the same
    tokens as the separate sampler on those logits, at temperature 0 and
    above."""
    k = 1024
    x, w = _operands(m, n, k, seed=m * 3 + n)
    x = (x.float() * 4).bfloat16()  # logits of a few units: near ties in the Gumbel scores
    g = torch.Generator(device="cpu").manual_seed(m + n)
    temps = torch.tensor([[0.0, 0.6, 1.0, 0.3][i % 4] for i in range(m)], dtype=torch.float32).cuda()
    seeds = torch.randint(0, 2**62, (m,), generator=g, dtype=torch.int64).cuda()
    plain = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    M_.layer_gemm(x, w, plain)
    want = torch.empty(m, dtype=torch.int32, device="cuda")
    M_.layer_sample(plain, temps, seeds, want)
    logits = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    got = torch.empty(m, dtype=torch.int32, device="cuda")
    M_.layer_gemm_sample(x, w, logits, temps, seeds, got)
    torch.cuda.synchronize()
    assert M_.gemm_device_error() == 0
    assert (bits(logits) == bits(plain)).all()
    assert got.tolist() == want.tolist()
