"""The C-ABI library loads on a machine without a GPU and exports every entry
point its headers declare; argument validation runs on the host before any
CUDA call, so it is testable here."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared(header):
    text = (ROOT / "include" / header).read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(nvbh?_[a-z0-9_]+)\s*\(", text)))


def exported(lib_path):
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True, check=True)
    return {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}


def test_kernel_library_exports_every_declared_symbol(nvb):
    names = declared("nvb_attention.h")
    assert "nvb_paged_fwd" in names and "nvb_qkv_rope_cached" in names
    syms = exported(nvb.LIB_PATH)
    missing = [n for n in names if n not in syms]
    assert not missing, missing
    lib = nvb.library()
    for n in names:
        assert hasattr(lib, n)


def test_num_splits_heuristic(nvb):
    # pure host function; invalid arguments return 0 like nvr_flash_num_splits
    assert nvb.num_splits(0, 16, 8, 4096, 148) == 0
    assert nvb.num_splits(4, 16, 5, 4096, 148) == 0
    assert nvb.num_splits(256, 32, 8, 4096, 148) == 1          # 2048 CTAs already fill the GPU
    assert nvb.num_splits(8, 16, 8, 4096, 148) == 4            # 64 CTAs x 4 = 256 fit one wave of 296
    assert nvb.num_splits(4, 64, 8, 32768, 148) == 9           # config 5 on one GPU: 288 CTAs, not 320
    assert nvb.num_splits(4, 8, 1, 32768, 148) == 74           # config 5 shard
    assert nvb.num_splits(1, 16, 8, 300, 148) == 2             # >= 256 keys per split
    assert 1 <= nvb.num_splits(1, 256, 1, 1 << 20, 148) <= 128


def _paged(lib, **kw):
    P = ctypes.c_void_p
    nz = P(256)  # any non-null, 16-byte aligned value: validation fails before use
    a = dict(batch=1, total_q=1, max_q=1, max_k=256, qh=4, kvh=2, bs=256, stride=1, splits=1, num_blocks=1)
    a.update(kw)
    return lib.nvb_paged_fwd_ex(P(0), nz, nz, nz, nz, nz, nz, nz, a["batch"], a["total_q"], a["max_q"], a["max_k"],
                                a["qh"], a["kvh"], a["bs"], a["stride"], a["splits"], nz, P(0), P(0), a["num_blocks"])


@pytest.mark.parametrize("bad", [dict(bs=128), dict(qh=5), dict(splits=129), dict(max_k=257), dict(batch=0),
                                 dict(max_q=2, splits=2), dict(total_q=2), dict(splits=2), dict(qh=512, kvh=2),
                                 dict(qh=34, kvh=2), dict(num_blocks=0)])
def test_paged_fwd_rejects_invalid_arguments_on_host(nvb, bad):
    lib = nvb.library()
    assert _paged(lib, **bad) == -1
    assert lib.nvb_last_error().decode()


def test_native_entry_rejects_unsupported_shapes_on_host(nvb):
    lib = nvb.library()
    P = ctypes.c_void_p
    nz = P(256)
    # head_dim beyond 512; block_size 2 at head_dim 128 (other head sizes run on
    # the generic path, which takes any block size)
    assert lib.nvb_attention(P(0), nz, nz, nz, nz, nz, nz, nz, 4, 4, 2, 600, 256, 4, 2, 2, 4096) == -1
    assert b"head_dim must be in [1, 512]" in lib.nvb_last_error()
    assert lib.nvb_attention(P(0), nz, nz, nz, nz, nz, nz, nz, 4, 4, 2, 128, 2, 4, 2, 2, 4096) == -1
    assert b"multiple of 32" in lib.nvb_last_error()
    assert lib.nvb_qkv_rope_cached(P(0), nz, nz, nz, nz, nz, nz, nz, nz, 1, 4, 2, 128, 256, 1, ctypes.c_float(0.0),
                                   nz, 16) == -1


def test_integration_notes_name_only_declared_entry_points():
    # Every C entry point that INTEGRATION.md tells a maintainer to bind (the
    # Rust extern block and the functions named in the text) is declared in
    # a header under include/.
    text = (ROOT / "INTEGRATION.md").read_text()
    named = set(re.findall(r"\bfn (nvb[a-z0-9_]*)\s*\(", text)) | set(re.findall(r"`(nvbe?h?_[a-z0-9_]+)`", text))
    declared_all = set()
    for h in (ROOT / "include").glob("*.h"):
        src = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        declared_all |= set(re.findall(r"\b(nvb[a-z]?_[a-z0-9_]+)\s*\(", src))
    assert named, "no entry points found in INTEGRATION.md"
    missing = sorted(n for n in named if n not in declared_all)
    assert not missing, missing
