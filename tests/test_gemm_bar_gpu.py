"""The tcgen05 decode GEMM timed beside cuBLAS on the same B200.

Qwen3-0.6B projection shapes (QKV 4096x1024, O 1024x2048, gate/up 6144x1024
with SiLU fused vs cuBLAS + the SiLU kernel, down 1024x3072, and the LM head
151936x1024 with the Gumbel-max sampler fused vs cuBLAS + the sampler) at decode batch
sizes, each side captured in a CUDA graph of back-to-back launches over
enough weight copies (> 200 MB) that the weights stream from HBM as in a
decode step. Where the model's dispatch (tc_gemms) picks this kernel, it must
not be slower than cuBLAS by more than 10 %. Setting NVB_GEMM_BAR_JSON=<path>
writes the figures there as JSON.
"""
import json
import os

import pytest
import torch

import __graft_entry__

pytestmark = pytest.mark.gpu

M_ = __graft_entry__.load_package().model
SHAPES = [("qkv", 4096, 1024, False), ("o", 1024, 2048, False), ("gate_up_silu", 6144, 1024, True),
          ("down", 1024, 3072, False)]
ROWS = [1, 8, 16, 32, 64, 128, 256]
PREFERRED = {  # the model's dispatch rule (gemm_decode_preferred)
    (name, m): (m <= 8 or (n <= 2048 and m <= 64)) for name, n, _, _ in SHAPES for m in ROWS}


def _graph_time(fn, copies, reps=4):
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(copies):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(copies * reps):
            fn(i % copies)
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) * 1000.0 / (copies * reps)


def test_decode_gemm_vs_cublas():
    results = {}
    gen = torch.Generator(device="cuda").manual_seed(0)
    for name, n, k, silu in SHAPES:
        copies = (256 << 20) // (n * k * 2) + 1
        ws_list = [(torch.randn(n, k, generator=gen, device="cuda") * 0.02).bfloat16() for _ in range(copies)]
        for m in ROWS:
            x = torch.randn(m, k, generator=gen, device="cuda").bfloat16()
            y = torch.empty(m, n // 2 if silu else n, dtype=torch.bfloat16, device="cuda")
            packed = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
            act = torch.empty(m, n // 2, dtype=torch.bfloat16, device="cuda")
            work = torch.empty(max(16, M_.gemm_workspace_bytes(m, n, k, silu)), dtype=torch.uint8, device="cuda")

            def mine(i):
                M_.layer_gemm(x, ws_list[i], y, silu=silu, workspace=work)

            def lib(i):
                torch.matmul(x, ws_list[i].t(), out=packed)
                if silu:
                    M_.layer_silu_mul(packed, act)

            t_mine, t_lib = _graph_time(mine, copies), _graph_time(lib, copies)
            results[f"{name}_m{m}"] = {"tcgen05_us": round(t_mine, 3), "cublas_us": round(t_lib, 3),
                                       "preferred": PREFERRED[(name, m)]}
        del ws_list
    # LM head (151936 x 1024) with the sampler fused vs cuBLAS + the sampler.
    n, k = 151936, 1024
    copies = 2
    heads = [(torch.randn(n, k, generator=gen, device="cuda") * 0.02).bfloat16() for _ in range(copies)]
    for m in (1, 4, 8, 16, 32):
        x = torch.randn(m, k, generator=gen, device="cuda").bfloat16()
        logits = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        temps = torch.full((m,), 0.6, dtype=torch.float32, device="cuda")
        seeds = torch.arange(m, dtype=torch.int64, device="cuda")
        toks = torch.empty(m, dtype=torch.int32, device="cuda")
        tiles = M_.library().nvbe_gemm_sample_tiles(n)
        ps = torch.empty(m * tiles, dtype=torch.float32, device="cuda")
        pi = torch.empty(m * tiles, dtype=torch.int32, device="cuda")
        parts = M_.library().nvbe_sample_partitions(n)
        ps2 = torch.empty(m * parts, dtype=torch.float32, device="cuda")
        pi2 = torch.empty(m * parts, dtype=torch.int32, device="cuda")
        lib_ = M_.library()

        def fused(i):
            lib_.nvbe_layer_gemm_sample(M_._s(None), M_._p(x), M_._p(heads[i]), M_._p(logits), m, n, k, M_._p(temps),
                                        M_._p(seeds), M_._p(toks), M_._p(ps), M_._p(pi))

        def separate(i):
            torch.matmul(x, heads[i].t(), out=logits)
            lib_.nvbe_layer_sample(M_._s(None), M_._p(logits), M_._p(temps), M_._p(seeds), M_._p(toks),
                                   M_._p(ps2), M_._p(pi2), m, n)

        t_f, t_s = _graph_time(fused, copies), _graph_time(separate, copies)
        results[f"lm_head_sample_m{m}"] = {"tcgen05_us": round(t_f, 3), "cublas_us": round(t_s, 3),
                                           "preferred": m <= 4}  # gemm_sample_preferred
    del heads
    assert M_.gemm_device_error() == 0
    path = os.environ.get("NVB_GEMM_BAR_JSON")
    if path:
        with open(path, "w") as f:
            json.dump(results, f, indent=1)
    slow = {k: v for k, v in results.items() if v["preferred"] and v["tcgen05_us"] > 1.10 * v["cublas_us"]}
    assert not slow, f"the dispatch picks the tcgen05 GEMM where cuBLAS is faster: {slow}"
