"""ctypes front-end of the CPU oracle (oracle.cpp) — TEST INFRASTRUCTURE ONLY.

Used by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, as
the checker or the timed CPU baseline. The library never imports this.
BF16 tensors cross this boundary as numpy uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
REF_NATIVE = HERE / "_ref" / "libref_native.so"
_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True)
        L = ctypes.CDLL(str(LIB))
        L.oracle_attention_native.argtypes = [_P] * 7 + [_I] * 10
        L.oracle_attention_varlen.argtypes = [_P] * 8 + [_I] * 8
        L.oracle_qkv_rope.argtypes = [_P] * 8 + [_I] * 6 + [ctypes.c_float, ctypes.c_float, _P, _I, _I]
        L.oracle_rope_cache.argtypes = [_P, _I, _I, ctypes.c_float]
        L.oracle_bf16_round.argtypes = [_P, _P, ctypes.c_longlong]
        L.oracle_hardware_threads.restype = _I
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return ctypes.c_void_p(a.ctypes.data)


def bf16_bits(x) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (src/gpu.rs:1151-1159)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_bf16_round(_p(x), _p(out), x.size)
    return out


def bits_to_f32(bits) -> np.ndarray:
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


def attention_native(q, k, v, positions, seqs, tables, *, qh, kvh, dim, bs, blocks, stride, batch, max_context,
                     threads=1):
    q = np.ascontiguousarray(q, dtype=np.uint16)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    positions, seqs, tables = i32(positions), i32(seqs), i32(tables)
    rows = positions.size
    out = np.zeros((rows, qh, dim), dtype=np.float32)
    lib().oracle_attention_native(_p(q), _p(k), _p(v), _p(positions), _p(seqs), _p(tables), _p(out), rows, qh, kvh,
                                  dim, bs, blocks, stride, batch, max_context, threads)
    return out


def attention_varlen(q, k, v, cu_q, kv_lens, table, *, qh, kvh, bs, blocks, stride, threads=1):
    """Returns (out [total_q, qh, 128] f32, lse [batch, qh, max_q] f32)."""
    q = np.ascontiguousarray(q, dtype=np.uint16)
    k = np.ascontiguousarray(k, dtype=np.uint16)
    v = np.ascontiguousarray(v, dtype=np.uint16)
    cu_q, kv_lens, table = i32(cu_q), i32(kv_lens), i32(table)
    batch = kv_lens.size
    max_q = int(np.max(np.diff(cu_q)))
    out = np.zeros((int(cu_q[-1]), qh, 128), dtype=np.float32)
    lse = np.full((batch, qh, max_q), -np.inf, dtype=np.float32)
    lib().oracle_attention_varlen(_p(q), _p(k), _p(v), _p(cu_q), _p(kv_lens), _p(table), _p(out), _p(lse), batch,
                                  max_q, qh, kvh, bs, blocks, stride, threads)
    return out, lse


def qkv_rope(qkv, qw, kw, positions, slots, qout, kcache, vcache, *, qh, kvh, dim, bs, blocks, eps, theta=1.0,
             rope_cache=None, max_positions=0):
    """Updates qout / kcache / vcache (uint16 arrays) in place."""
    qkv = np.ascontiguousarray(qkv, dtype=np.uint16)
    qw = np.ascontiguousarray(qw, dtype=np.uint16)
    kw = np.ascontiguousarray(kw, dtype=np.uint16)
    positions, slots = i32(positions), i32(slots)
    for a in (qout, kcache, vcache):
        assert a.dtype == np.uint16 and a.flags["C_CONTIGUOUS"]
    cached = rope_cache is not None
    rc = np.ascontiguousarray(rope_cache, dtype=np.float32) if cached else np.zeros(1, np.float32)
    lib().oracle_qkv_rope(_p(qkv), _p(qw), _p(kw), _p(positions), _p(slots), _p(qout), _p(kcache), _p(vcache),
                          positions.size, qh, kvh, dim, bs, blocks, eps, theta, _p(rc), max_positions, int(cached))


def rope_cache(positions, dim, theta):
    out = np.zeros((positions, dim), dtype=np.float32)
    lib().oracle_rope_cache(_p(out), positions, dim, theta)
    return out


def hardware_threads() -> int:
    return int(lib().oracle_hardware_threads())
