"""Python binding of the B200 paged-attention library (libnvb.so).

This mirrors the checked wrappers the reference's Rust device layer puts in
front of its C ABI (src/gpu.rs:482-509 tensor extents / alignment / aliasing,
src/gpu.rs:775-995 qkv_rope_cached, paged_attention and flash_attention),
for torch tensors. Every call goes through the C ABI declared in
include/nvb_attention.h; there is no CPU or PyTorch fallback: if the CUDA
library is missing, loading fails loudly.

The package directory is named ``nano-vllm-rs_b200`` (not importable with a
plain ``import``); load it with ``__graft_entry__.load_package()`` which
registers it as ``nano_vllm_rs_b200``.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_DIR = PKG_DIR / "_lib"
LIB_PATH = LIB_DIR / "libnvb.so"
HOST_LIB_PATH = LIB_DIR / "libnvb_host.so"
INCLUDE_DIR = PKG_DIR.parent / "include"

_lib = None
_host = None

c_int, c_float, c_void_p, c_char_p = ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_char_p
_P = c_void_p


def _declare(lib):
    sig = {
        "nvb_paged_fwd": [_P] * 8 + [c_int] * 9 + [_P] * 3,
        "nvb_paged_fwd_ex": [_P] * 8 + [c_int] * 9 + [_P] * 3 + [c_int],
        "nvb_num_splits": [c_int] * 5,
        "nvb_attention": [_P] * 8 + [c_int] * 9,
        "nvb_attention_splitkv": [_P] * 8 + [c_int] * 9 + [_P, c_int],
        "nvb_qkv_rope_cached": [_P] * 9 + [c_int] * 6 + [c_float, _P, c_int],
        "nvb_qkv_rope": [_P] * 9 + [c_int] * 6 + [c_float, c_float],
        "nvb_rope_cache": [_P, _P, c_int, c_int, c_float],
        "nvb_capture_begin": [_P],
        "nvb_capture_end": [_P, ctypes.POINTER(c_void_p)],
        "nvb_capture_abort": [_P],
        "nvb_graph_replay": [_P, _P],
        "nvb_graph_destroy": [_P],
        "nvb_device_error": [ctypes.POINTER(c_int)],
        "nvb_clear_device_error": [],
        "nvb_paged_decode_gather": [_P] * 8 + [c_int] * 8 + [_P] * 4 + [c_int, c_int, ctypes.c_uint],
        "nvb_paged_decode_gather_capturable": [_P] * 8 + [c_int] * 8 + [_P] * 5 + [c_int, c_int],
        "nvb_peer_buffer_create": [ctypes.c_size_t, ctypes.POINTER(c_void_p), _P],
        "nvb_peer_buffer_open": [_P, ctypes.POINTER(c_void_p)],
        "nvb_peer_buffer_close": [_P],
        "nvb_peer_buffer_free": [_P],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = None if name in ("nvb_capture_abort", "nvb_graph_destroy") else c_int
    for name in ("nvb_last_error", "nvb_version"):
        getattr(lib, name).restype = c_char_p
        getattr(lib, name).argtypes = []


def library():
    """Loads libnvb.so (built by ``build.py``); raises if it is missing."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() first")
        lib = ctypes.CDLL(str(LIB_PATH))
        _declare(lib)
        _lib = lib
    return _lib


class NvbError(RuntimeError):
    pass


def _check(code: int):
    if code != 0:
        msg = library().nvb_last_error().decode(errors="replace")
        raise NvbError(f"libnvb: {msg} (status {code})")


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream(stream=None):
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _tensor(t, shape, dtype, name):
    """Extent/dtype/contiguity check, like Gpu::tensor (src/gpu.rs:482-501)."""
    if t is None:
        raise NvbError(f"{name} is required")
    if not t.is_cuda:
        raise NvbError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise NvbError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise NvbError(f"{name} must be contiguous")
    need = 1
    for d in shape:
        need *= int(d)
    if t.numel() < need:
        raise NvbError(f"{name} has {t.numel()} elements, needs {need} for shape {tuple(shape)}")


def _span(t):
    start = t.data_ptr()
    return start, start + t.numel() * t.element_size()


def _distinct(output, inputs, name):
    """Rejects an output that overlaps an input (src/gpu.rs:502-509)."""
    o0, o1 = _span(output)
    for t in inputs:
        if t is None:
            continue
        a0, a1 = _span(t)
        if o0 < a1 and a0 < o1:
            raise NvbError(f"{name} aliases an input or another output")


def num_splits(batch, q_heads, kv_heads, max_k, num_sms):
    return library().nvb_num_splits(batch, q_heads, kv_heads, max_k, num_sms)


def splitkv_scratch(num_splits_, batch, q_heads, device):
    """Caller-owned FP32 split-KV scratch (lse_accum, out_accum)."""
    import torch

    lse_accum = torch.empty(num_splits_, batch, q_heads, dtype=torch.float32, device=device)
    out_accum = torch.empty(num_splits_, batch, q_heads, 128, dtype=torch.float32, device=device)
    return lse_accum, out_accum


def peer_buffer_create(nbytes):
    """A zeroed device buffer of this GPU to share with the node's other ranks:
    returns (device pointer, 64-byte CUDA IPC handle)."""
    ptr = c_void_p()
    handle = ctypes.create_string_buffer(64)
    _check(library().nvb_peer_buffer_create(nbytes, ctypes.byref(ptr), handle))
    return ptr.value, handle.raw


def peer_buffer_open(handle):
    """Maps another rank's buffer (its IPC handle) into this process."""
    ptr = c_void_p()
    buf = ctypes.create_string_buffer(bytes(handle), 64)
    _check(library().nvb_peer_buffer_open(buf, ctypes.byref(ptr)))
    return ptr.value


def peer_buffer_close(ptr):
    _check(library().nvb_peer_buffer_close(c_void_p(ptr)))


def peer_buffer_free(ptr):
    _check(library().nvb_peer_buffer_free(c_void_p(ptr)))


def paged_decode_gather(q, k, v, out_local, cu_q, kv_lens, block_table, *, batch, max_k, q_heads, kv_heads,
                        block_size, table_stride, num_blocks, num_splits, lse_accum, out_accum, peer_out, peer_flag,
                        rank, epoch, stream=None, check=True):
    """Decode of this rank's kv heads with the combine fused into the
    all-gather of the outputs (nvb_paged_decode_gather): `peer_out` and
    `peer_flag` are every rank's output and flag device pointers (ints)."""
    import torch

    world = len(peer_out)
    if check:
        _tensor(q, (batch, q_heads, 128), torch.bfloat16, "q")
        _tensor(out_local, (batch, q_heads, 128), torch.bfloat16, "out_local")
        for t, nm in ((k, "k"), (v, "v")):
            _tensor(t, (num_blocks, block_size, kv_heads, 128), torch.bfloat16, nm)
        _tensor(cu_q, (batch + 1,), torch.int32, "cu_q")
        _tensor(kv_lens, (batch,), torch.int32, "kv_lens")
        _tensor(block_table, (batch, table_stride), torch.int32, "block_table")
        if num_splits > 1:
            _tensor(lse_accum, (num_splits, batch, q_heads), torch.float32, "lse_accum")
            _tensor(out_accum, (num_splits, batch, q_heads, 128), torch.float32, "out_accum")
        if len(peer_flag) != world or not 1 <= world <= 8:
            raise ValueError("peer_out and peer_flag need one pointer per rank (1..8 ranks)")
    outs = (c_void_p * world)(*peer_out)
    flags = (c_void_p * world)(*peer_flag)
    _check(library().nvb_paged_decode_gather(
        _stream(stream), _ptr(q), _ptr(k), _ptr(v), _ptr(out_local), _ptr(cu_q), _ptr(kv_lens), _ptr(block_table),
        batch, max_k, q_heads, kv_heads, block_size, table_stride, num_blocks, num_splits, _ptr(lse_accum),
        _ptr(out_accum), ctypes.cast(outs, c_void_p), ctypes.cast(flags, c_void_p), world, rank, epoch))


def paged_decode_gather_capturable(q, k, v, out_local, cu_q, kv_lens, block_table, *, batch, max_k, q_heads,
                                   kv_heads, block_size, table_stride, num_blocks, num_splits, lse_accum, out_accum,
                                   peer_out0, peer_out1, peer_flag, rank, stream=None, check=True):
    """nvb_paged_decode_gather_capturable: the same step with the epoch kept
    in device memory (slot len(peer_flag) of this rank's flags), so that a
    CUDA graph can capture it once; step n writes output set n & 1
    (`peer_out1` for odd n)."""
    import torch

    world = len(peer_out0)
    if check:
        _tensor(q, (batch, q_heads, 128), torch.bfloat16, "q")
        _tensor(out_local, (batch, q_heads, 128), torch.bfloat16, "out_local")
        for t, nm in ((k, "k"), (v, "v")):
            _tensor(t, (num_blocks, block_size, kv_heads, 128), torch.bfloat16, nm)
        _tensor(cu_q, (batch + 1,), torch.int32, "cu_q")
        _tensor(kv_lens, (batch,), torch.int32, "kv_lens")
        _tensor(block_table, (batch, table_stride), torch.int32, "block_table")
        if num_splits > 1:
            _tensor(lse_accum, (num_splits, batch, q_heads), torch.float32, "lse_accum")
            _tensor(out_accum, (num_splits, batch, q_heads, 128), torch.float32, "out_accum")
        if len(peer_out1) != world or len(peer_flag) != world or not 1 <= world <= 8:
            raise ValueError("peer_out0, peer_out1 and peer_flag need one pointer per rank (1..8 ranks)")
    o0 = (c_void_p * world)(*peer_out0)
    o1 = (c_void_p * world)(*peer_out1)
    flags = (c_void_p * world)(*peer_flag)
    _check(library().nvb_paged_decode_gather_capturable(
        _stream(stream), _ptr(q), _ptr(k), _ptr(v), _ptr(out_local), _ptr(cu_q), _ptr(kv_lens), _ptr(block_table),
        batch, max_k, q_heads, kv_heads, block_size, table_stride, num_blocks, num_splits, _ptr(lse_accum),
        _ptr(out_accum), ctypes.cast(o0, c_void_p), ctypes.cast(o1, c_void_p), ctypes.cast(flags, c_void_p), world,
        rank))


def paged_fwd(q, k, v, out, cu_q, kv_lens, block_table, *, batch, max_q, max_k, q_heads, kv_heads,
              block_size, table_stride, num_blocks, num_splits=1, lse=None, lse_accum=None,
              out_accum=None, stream=None, check=True):
    """Paged attention through nvb_paged_fwd_ex (the bounded entry point).

    Same argument meaning as the reference's Gpu::flash_attention
    (src/gpu.rs:890-995) / nvr_flash_fwd.
    """
    import torch

    total_q = q.shape[0]
    if check:
        for t, nm in ((q, "q"), (out, "out")):
            _tensor(t, (total_q, q_heads, 128), torch.bfloat16, nm)
        for t, nm in ((k, "k"), (v, "v")):
            _tensor(t, (num_blocks, block_size, kv_heads, 128), torch.bfloat16, nm)
        _tensor(cu_q, (batch + 1,), torch.int32, "cu_q")
        _tensor(kv_lens, (batch,), torch.int32, "kv_lens")
        _tensor(block_table, (batch, table_stride), torch.int32, "block_table")
        if lse is not None:
            _tensor(lse, (batch, q_heads, max_q), torch.float32, "lse")
        if num_splits > 1:
            _tensor(lse_accum, (num_splits, batch, q_heads), torch.float32, "lse_accum")
            _tensor(out_accum, (num_splits, batch, q_heads, 128), torch.float32, "out_accum")
        inputs = [q, k, v, cu_q, kv_lens, block_table]
        outputs = [out, lse, lse_accum, out_accum]
        for i, o in enumerate(outputs):
            if o is not None:
                _distinct(o, inputs + [x for x in outputs[:i] if x is not None], "output")
    lib = library()
    _check(lib.nvb_paged_fwd_ex(_stream(stream), _ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(cu_q),
                                _ptr(kv_lens), _ptr(block_table), batch, total_q, max_q, max_k, q_heads,
                                kv_heads, block_size, table_stride, num_splits, _ptr(lse), _ptr(lse_accum),
                                _ptr(out_accum), num_blocks))


def attention(q, kcache, vcache, positions, seq_indices, tables, out, *, rows, q_heads, kv_heads, head_dim,
              block_size, num_blocks, table_stride, batch, max_context, scratch=None, partitions=1,
              stream=None):
    """Native-form paged attention (Gpu::paged_attention, src/gpu.rs:829-887)."""
    import torch

    _tensor(q, (rows, q_heads, head_dim), torch.bfloat16, "q")
    _tensor(out, (rows, q_heads, head_dim), torch.bfloat16, "out")
    for t, nm in ((kcache, "kcache"), (vcache, "vcache")):
        _tensor(t, (num_blocks, block_size, kv_heads, head_dim), torch.bfloat16, nm)
    _tensor(positions, (rows,), torch.int32, "positions")
    _tensor(seq_indices, (rows,), torch.int32, "seq_indices")
    _tensor(tables, (batch, table_stride), torch.int32, "tables")
    _distinct(out, [q, kcache, vcache, positions, seq_indices, tables], "out")
    lib = library()
    if partitions > 1:
        _tensor(scratch, (rows * q_heads * partitions * (head_dim + 2),), torch.float32, "scratch")
        _check(lib.nvb_attention_splitkv(_stream(stream), _ptr(q), _ptr(kcache), _ptr(vcache), _ptr(positions),
                                         _ptr(seq_indices), _ptr(tables), _ptr(out), rows, q_heads, kv_heads,
                                         head_dim, block_size, num_blocks, table_stride, batch, max_context,
                                         _ptr(scratch), partitions))
    else:
        _check(lib.nvb_attention(_stream(stream), _ptr(q), _ptr(kcache), _ptr(vcache), _ptr(positions),
                                 _ptr(seq_indices), _ptr(tables), _ptr(out), rows, q_heads, kv_heads, head_dim,
                                 block_size, num_blocks, table_stride, batch, max_context))


def qkv_rope_cached(qkv, q_weight, k_weight, positions, slots, qout, kcache, vcache, *, rows, q_heads, kv_heads,
                    head_dim, block_size, num_blocks, eps, rope_cache, max_positions, stream=None, check=True):
    """Fused norm + RoPE + KV store (Gpu::qkv_rope_cached, src/gpu.rs:775-825)."""
    import torch

    if check:
        _tensor(qkv, (rows, q_heads + 2 * kv_heads, head_dim), torch.bfloat16, "qkv")
        _tensor(q_weight, (head_dim,), torch.bfloat16, "q_weight")
        _tensor(k_weight, (head_dim,), torch.bfloat16, "k_weight")
        _tensor(positions, (rows,), torch.int32, "positions")
        _tensor(slots, (rows,), torch.int32, "slots")
        _tensor(qout, (rows, q_heads, head_dim), torch.bfloat16, "qout")
        for t, nm in ((kcache, "kcache"), (vcache, "vcache")):
            _tensor(t, (num_blocks, block_size, kv_heads, head_dim), torch.bfloat16, nm)
        _tensor(rope_cache, (max_positions, head_dim), torch.float32, "rope_cache")
        inputs = [qkv, q_weight, k_weight, positions, slots, rope_cache]
        _distinct(qout, inputs + [kcache, vcache], "qout")
        _distinct(kcache, inputs + [vcache], "kcache")
        _distinct(vcache, inputs, "vcache")
    _check(library().nvb_qkv_rope_cached(_stream(stream), _ptr(qkv), _ptr(q_weight), _ptr(k_weight),
                                         _ptr(positions), _ptr(slots), _ptr(qout), _ptr(kcache), _ptr(vcache),
                                         rows, q_heads, kv_heads, head_dim, block_size, num_blocks, float(eps),
                                         _ptr(rope_cache), max_positions))


def qkv_rope(qkv, q_weight, k_weight, positions, slots, qout, kcache, vcache, *, rows, q_heads, kv_heads, head_dim,
             block_size, num_blocks, eps, theta, stream=None):
    """Fused norm + RoPE + KV store with in-kernel angles (nv_qkv_rope)."""
    _check(library().nvb_qkv_rope(_stream(stream), _ptr(qkv), _ptr(q_weight), _ptr(k_weight), _ptr(positions),
                                  _ptr(slots), _ptr(qout), _ptr(kcache), _ptr(vcache), rows, q_heads, kv_heads,
                                  head_dim, block_size, num_blocks, float(eps), float(theta)))


def rope_cache(cache, positions, head_dim, theta, stream=None):
    import torch

    _tensor(cache, (positions, head_dim), torch.float32, "rope_cache")
    _check(library().nvb_rope_cache(_stream(stream), _ptr(cache), positions, head_dim, float(theta)))


def device_error():
    code = c_int(0)
    _check(library().nvb_device_error(ctypes.byref(code)))
    return code.value


def clear_device_error():
    _check(library().nvb_clear_device_error())


class Graph:
    """A captured CUDA graph (mirrors Gpu::capture / Graph, src/gpu.rs:511-533,
    1128-1146). Keeps references to the tensors the capture used so their
    memory outlives the graph."""

    def __init__(self, handle, keep):
        self._handle = handle
        self._keep = keep

    def replay(self, stream=None):
        _check(library().nvb_graph_replay(self._handle, _stream(stream)))

    def close(self):
        if self._handle:
            library().nvb_graph_destroy(self._handle)
            self._handle = None
            self._keep = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def capture(fn, keep=(), stream=None):
    """Captures the device work `fn()` enqueues on `stream` into a Graph."""
    s = _stream(stream)
    lib = library()
    _check(lib.nvb_capture_begin(s))
    try:
        fn()
    except BaseException:
        lib.nvb_capture_abort(s)
        raise
    handle = ctypes.c_void_p(0)
    _check(lib.nvb_capture_end(s, ctypes.byref(handle)))
    return Graph(handle, list(keep))


def version():
    return library().nvb_version().decode()


from . import workloads  # noqa: E402  (seeded benchmark inputs)
from . import engine  # noqa: E402,F401  (continuous-batching scheduler, libnvb_host.so)
from . import model  # noqa: E402,F401  (Qwen3 runner, libnvb_model.so)
