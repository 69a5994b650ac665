"""Shared fixtures. GPU tests are marked ``gpu``; everything else runs on CPU."""
from __future__ import annotations

import ctypes
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT / "tests"))

import __graft_entry__  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a)")


@pytest.fixture(scope="session")
def nvb():
    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def oracle():
    import oracle as o  # oracle/oracle.py

    return o


def bits(t) -> np.ndarray:
    """torch bf16 tensor -> numpy uint16 bit patterns (on the host)."""
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def as_f32(t) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def assert_close(actual, expected, max_abs, mean_abs, what=""):
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape, (actual.shape, expected.shape)
    assert np.all(np.isfinite(actual)), f"{what}: non-finite output"
    err = np.abs(actual - expected)
    mx, mn = float(err.max(initial=0.0)), float(err.mean()) if err.size else 0.0
    assert mx <= max_abs and mn <= mean_abs, f"{what}: max-abs {mx:.3g} (<= {max_abs}), mean-abs {mn:.3g} (<= {mean_abs})"
    return mx, mn


class RefNative:
    """The reference's own CUDA kernels (oracle/_ref/libref_native.so, built from
    kernels/kernels.cu + kernels/decode_candidate.cuh) behind their nv_* ABI."""

    def __init__(self, path):
        L = ctypes.CDLL(str(path))
        P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.nv_create.argtypes = [I, ctypes.POINTER(P)]
        L.nv_stream.argtypes = [P, ctypes.POINTER(P)]
        L.nv_sync.argtypes = [P]
        L.nv_destroy.argtypes = [P]
        L.nv_destroy.restype = None
        L.nv_last_error.restype = ctypes.c_char_p
        L.nv_attention.argtypes = [P] * 8 + [I] * 9
        L.nv_attention_splitkv_candidate.argtypes = [P] * 8 + [I] * 9 + [P, I]
        L.nv_qkv_rope_cached.argtypes = [P] * 9 + [I] * 6 + [F, P, I]
        L.nv_qkv_rope.argtypes = [P] * 9 + [I] * 6 + [F, F]
        L.nv_rope_cache.argtypes = [P, P, I, I, F]
        self.L = L
        ctx = P()
        self._check(L.nv_create(0, ctypes.byref(ctx)))
        self.ctx = ctx

    def _check(self, code):
        if code:
            raise RuntimeError(f"reference kernel: {self.L.nv_last_error().decode()} ({code})")

    def sync(self):
        self._check(self.L.nv_sync(self.ctx))

    def call(self, name, *args):
        conv = [ctypes.c_void_p(a.data_ptr()) if hasattr(a, "data_ptr") else a for a in args]
        self._check(getattr(self.L, name)(self.ctx, *conv))
        self.sync()


@pytest.fixture(scope="session")
def ref_native():
    import torch

    path = ROOT / "oracle" / "_ref" / "libref_native.so"
    if not path.exists():
        pytest.skip("reference kernels were not built (oracle/_ref)")
    torch.cuda.synchronize()
    return RefNative(path)


@pytest.fixture(scope="session")
def ref_flash():
    """The reference's FA2 adapter (oracle/_ref/libref_flash.so, built from
    kernels/flash_native/flash_native.cu and its vendored FA2 / CUTLASS)."""
    path = ROOT / "oracle" / "_ref" / "libref_flash.so"
    if not path.exists():
        pytest.skip("the reference FA2 adapter was not built (oracle/_ref)")
    P, I = ctypes.c_void_p, ctypes.c_int
    L = ctypes.CDLL(str(path))
    L.nvr_flash_fwd.argtypes = [P] * 8 + [I] * 9 + [P] * 3
    L.nvr_flash_fwd.restype = I
    L.nvr_flash_num_splits.argtypes = [I] * 5
    L.nvr_flash_num_splits.restype = I
    L.nvr_flash_last_error.restype = ctypes.c_char_p
    return L


@pytest.fixture(autouse=True)
def _gpu_guard(request):
    if request.node.get_closest_marker("gpu"):
        import torch

        if not torch.cuda.is_available():
            pytest.skip("needs a CUDA device")
    yield
