"""Writes tests/golden/*.npz from the reference's own CUDA kernels.

Run on a B200 from the repository root after `make -C oracle`:
    python tests/golden/make_golden.py [output_dir]   (default: tests/golden)
It loads oracle/_ref/libref_native.so (kernels/kernels.cu and
kernels/decode_candidate.cuh compiled from the reference sources), runs
nv_attention, nv_attention_splitkv_candidate, nv_rope_cache and
nv_qkv_rope_cached on the hashed inputs of tests/golden_check.py, and stores
their outputs.
"""
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT / "tests"), str(ROOT / "oracle"), str(ROOT)]

import golden_check as G  # noqa: E402
import oracle  # noqa: E402
from conftest import RefNative  # noqa: E402


def dev(a):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    return torch.from_numpy(a).cuda()


def host_bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def main():
    ref = RefNative(ROOT / "oracle" / "_ref" / "libref_native.so")
    out_dir = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent
    out_dir.mkdir(parents=True, exist_ok=True)
    q, k, v, pos, seqs, tbl = G.attention_inputs(oracle)
    rows = len(pos)
    dq, dk, dv, dp, ds, dt = dev(q), dev(k), dev(v), dev(pos), dev(seqs), dev(tbl)
    out = torch.zeros(rows, G.QH, G.DIM, dtype=torch.bfloat16, device="cuda")
    ref.call("nv_attention", dq, dk, dv, dp, ds, dt, out, rows, G.QH, G.KVH, G.DIM, G.BS, G.NUM_BLOCKS, G.STRIDE,
             len(G.PAGES), 4096)
    parts = 4
    scratch = torch.zeros(rows * G.QH * parts * (G.DIM + 2), dtype=torch.float32, device="cuda")
    sout = torch.zeros_like(out)
    ref.call("nv_attention_splitkv_candidate", dq, dk, dv, dp, ds, dt, sout, rows, G.QH, G.KVH, G.DIM, G.BS,
             G.NUM_BLOCKS, G.STRIDE, len(G.PAGES), 4096, scratch, parts)
    np.savez_compressed(out_dir / "native_attention.npz", out=host_bits(out), splitkv_out=host_bits(sout))

    table = torch.zeros(G.MAXPOS, G.DIM, dtype=torch.float32, device="cuda")
    ref.call("nv_rope_cache", table, G.MAXPOS, G.DIM, G.THETA)
    qkv, qw, kw, p, s = G.rope_inputs(oracle)
    qout = torch.zeros(G.ROPE_ROWS, G.QH, G.DIM, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(G.ROPE_BLOCKS, G.BS, G.KVH, G.DIM, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    ref.call("nv_qkv_rope_cached", dev(qkv), dev(qw), dev(kw), dev(p), dev(s), qout, kc, vc, G.ROPE_ROWS, G.QH,
             G.KVH, G.DIM, G.BS, G.ROPE_BLOCKS, G.EPS, table, G.MAXPOS)
    valid = (s >= 0) & (s < G.ROPE_BLOCKS * G.BS)
    idx = torch.from_numpy(s[valid].astype(np.int64)).cuda()
    np.savez_compressed(out_dir / "qkv_rope.npz", qout=host_bits(qout),
                        k_slots=host_bits(kc.view(-1, G.KVH, G.DIM)[idx]),
                        v_slots=host_bits(vc.view(-1, G.KVH, G.DIM)[idx]),
                        rope_rows=table[torch.from_numpy(G.TABLE_ROWS_SAMPLED.astype(np.int64)).cuda()].cpu().numpy())
    print("wrote", sorted(p.name for p in out_dir.glob("*.npz")))


if __name__ == "__main__":
    main()
