"""ctypes binding of libnvb_host.so (include/nvb_host.h): the host-side
integer metadata of the paged attention path, runnable without a GPU."""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libnvb_host.so"
_lib = None

c_size = ctypes.c_size_t
P = ctypes.c_void_p


class NvbhBatch(ctypes.Structure):
    _fields_ = [("token_ids", P), ("positions", P), ("sequence_ids", P), ("slot_mapping", P), ("rows", c_size),
                ("block_tables", P), ("block_tables_len", c_size), ("table_stride", c_size),
                ("last_token_indices", P), ("temperatures", P), ("seeds", P), ("samples", c_size),
                ("is_decode", ctypes.c_int)]


class NvbhMetadataLayout(ctypes.Structure):
    _fields_ = [("start", c_size * 10), ("end", c_size * 10), ("bytes", c_size)]


class NvbhLimits(ctypes.Structure):
    _fields_ = [(n, c_size) for n in ("max_batch_tokens", "max_sequences", "max_model_len", "block_size",
                                      "num_blocks", "table_stride", "vocab_size")]


class NvbhSegment(ctypes.Structure):
    _fields_ = [("tokens", P), ("num_tokens", c_size), ("blocks", P), ("num_blocks", c_size), ("start", c_size),
                ("end", c_size), ("sample", ctypes.c_int), ("request_id", ctypes.c_uint64),
                ("generated", c_size), ("temperature", ctypes.c_float)]


class NvbhBatchOut(ctypes.Structure):
    _fields_ = [("token_ids", P), ("positions", P), ("sequence_ids", P), ("slot_mapping", P), ("rows_cap", c_size),
                ("block_tables", P), ("tables_cap", c_size), ("last_token_indices", P), ("temperatures", P),
                ("seeds", P), ("samples_cap", c_size), ("rows", c_size), ("table_stride", c_size),
                ("samples", c_size)]


FIELDS = ["tokens", "positions", "sequences", "slots", "tables", "last_indices", "temperatures", "seeds", "cu_q",
          "kv_lens"]


def library():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build() first")
        L = ctypes.CDLL(str(LIB_PATH))
        L.nvbh_last_error.restype = ctypes.c_char_p
        L.nvbh_flash_metadata.argtypes = [P, P, c_size, c_size, P, P, ctypes.POINTER(c_size)]
        L.nvbh_metadata_layout.argtypes = [c_size, c_size, c_size, ctypes.POINTER(NvbhMetadataLayout)]
        L.nvbh_metadata_pack.argtypes = [ctypes.POINTER(NvbhMetadataLayout), P, c_size, ctypes.POINTER(NvbhBatch),
                                         c_size, c_size, P, P]
        L.nvbh_validate_batch.argtypes = [ctypes.POINTER(NvbhBatch), ctypes.POINTER(NvbhLimits),
                                          ctypes.POINTER(c_size), ctypes.POINTER(c_size), ctypes.POINTER(c_size)]
        L.nvbh_pool_create.restype = P
        L.nvbh_pool_create.argtypes = [c_size]
        L.nvbh_pool_destroy.argtypes = [P]
        L.nvbh_pool_destroy.restype = None
        for n in ("allocate",):
            getattr(L, f"nvbh_pool_{n}").argtypes = [P]
        L.nvbh_pool_release.argtypes = [P, ctypes.c_int]
        L.nvbh_pool_release.restype = None
        L.nvbh_pool_find.argtypes = [P, P, c_size]
        L.nvbh_pool_find_and_retain.argtypes = [P, P, c_size]
        L.nvbh_pool_publish.argtypes = [P, ctypes.c_int, P, c_size]
        L.nvbh_pool_publish.restype = None
        for n in ("available", "in_use", "cached_keys"):
            getattr(L, f"nvbh_pool_{n}").argtypes = [P]
            getattr(L, f"nvbh_pool_{n}").restype = c_size
        L.nvbh_pool_references.argtypes = [P, ctypes.c_int]
        L.nvbh_pool_references.restype = c_size
        L.nvbh_pool_clear_cache.argtypes = [P]
        L.nvbh_pool_clear_cache.restype = None
        L.nvbh_pool_force_hash_entry.argtypes = [P, P, c_size, ctypes.c_int]
        L.nvbh_pool_force_hash_entry.restype = None
        L.nvbh_make_batch.argtypes = [ctypes.POINTER(NvbhSegment), c_size, c_size, ctypes.c_uint64,
                                      ctypes.POINTER(NvbhBatchOut)]
        L.nvbh_sampling_seed.argtypes = [ctypes.c_uint64] * 3
        L.nvbh_sampling_seed.restype = ctypes.c_uint64
        _lib = L
    return _lib


class HostError(ValueError):
    pass


def _check(rc):
    if rc != 0:
        raise HostError(library().nvbh_last_error().decode())


def _arr(values, dtype):
    return np.ascontiguousarray(np.asarray(values, dtype=dtype))


def _p(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None and a.size else ctypes.c_void_p(0)


@dataclass
class Batch:
    """The reference's Batch (src/runtime.rs:17-29)."""
    token_ids: list = field(default_factory=list)
    positions: list = field(default_factory=list)
    sequence_ids: list = field(default_factory=list)
    slot_mapping: list = field(default_factory=list)
    block_tables: list = field(default_factory=list)
    table_stride: int = 0
    last_token_indices: list = field(default_factory=list)
    temperatures: list = field(default_factory=list)
    seeds: list = field(default_factory=list)
    is_decode: bool = False

    def to_c(self):
        arrays = dict(token_ids=_arr(self.token_ids, np.int32), positions=_arr(self.positions, np.int32),
                      sequence_ids=_arr(self.sequence_ids, np.int32), slot_mapping=_arr(self.slot_mapping, np.int32),
                      block_tables=_arr(self.block_tables, np.int32),
                      last_token_indices=_arr(self.last_token_indices, np.int32),
                      temperatures=_arr(self.temperatures, np.float32), seeds=_arr(self.seeds, np.uint64))
        rows = len(self.positions)
        c = NvbhBatch(_p(arrays["token_ids"]) if len(self.token_ids) == rows else None, _p(arrays["positions"]),
                      _p(arrays["sequence_ids"]), _p(arrays["slot_mapping"]) if len(self.slot_mapping) == rows else None,
                      rows, _p(arrays["block_tables"]), len(self.block_tables), self.table_stride,
                      _p(arrays["last_token_indices"]), _p(arrays["temperatures"]), _p(arrays["seeds"]),
                      len(self.last_token_indices), int(self.is_decode))
        return c, arrays


def flash_metadata(batch: Batch, sequences: int):
    """(cu_q, kv_lens, max_q) as src/model.rs:234-267."""
    pos = _arr(batch.positions, np.int32)
    seq = _arr(batch.sequence_ids, np.int32)
    cu = np.zeros(sequences + 1, np.int32)
    kv = np.zeros(max(sequences, 1), np.int32)
    mq = c_size(0)
    _check(library().nvbh_flash_metadata(_p(pos), _p(seq), pos.size, sequences, _p(cu), _p(kv), ctypes.byref(mq)))
    return cu.tolist(), kv[:sequences].tolist(), mq.value


class MetadataLayout:
    """The packed metadata upload ranges (src/model.rs:271-358)."""

    def __init__(self, tokens, sequences, table_stride):
        self.c = NvbhMetadataLayout()
        _check(library().nvbh_metadata_layout(tokens, sequences, table_stride, ctypes.byref(self.c)))
        self.bytes = self.c.bytes
        self.ranges = {f: (self.c.start[i], self.c.end[i]) for i, f in enumerate(FIELDS)}

    def pack(self, staging: np.ndarray, batch: Batch, sequences, table_stride, cu_q=None, kv_lens=None):
        assert staging.dtype == np.uint8 and staging.flags["C_CONTIGUOUS"]
        cb, keep = batch.to_c()
        cu = _arr(cu_q, np.int32) if cu_q is not None else None
        kv = _arr(kv_lens, np.int32) if kv_lens is not None else None
        _check(library().nvbh_metadata_pack(ctypes.byref(self.c), _p(staging), staging.size, ctypes.byref(cb),
                                            sequences, table_stride, _p(cu) if cu is not None else None,
                                            _p(kv) if kv is not None else None))
        del keep


def validate_batch(batch: Batch, *, max_batch_tokens, max_sequences, max_model_len, block_size, num_blocks,
                   table_stride, vocab_size):
    """(rows, sequences, samples) or HostError, as src/model.rs:820-921."""
    cb, keep = batch.to_c()
    lim = NvbhLimits(max_batch_tokens, max_sequences, max_model_len, block_size, num_blocks, table_stride, vocab_size)
    r, s, k = c_size(0), c_size(0), c_size(0)
    _check(library().nvbh_validate_batch(ctypes.byref(cb), ctypes.byref(lim), ctypes.byref(r), ctypes.byref(s),
                                         ctypes.byref(k)))
    del keep
    return r.value, s.value, k.value


class BlockPool:
    """Reference-counted page pool with exact prefix keys (src/runtime.rs:192-296)."""

    def __init__(self, num_blocks):
        self.h = library().nvbh_pool_create(num_blocks)

    def __del__(self):
        if getattr(self, "h", None):
            library().nvbh_pool_destroy(self.h)
            self.h = None

    def _toks(self, tokens):
        return _arr(tokens, np.uint32)

    def allocate(self):
        b = library().nvbh_pool_allocate(self.h)
        return None if b < 0 else b

    def release(self, block):
        library().nvbh_pool_release(self.h, block)

    def find(self, tokens):
        t = self._toks(tokens)
        b = library().nvbh_pool_find(self.h, _p(t), t.size)
        return None if b < 0 else b

    def find_and_retain(self, tokens):
        t = self._toks(tokens)
        b = library().nvbh_pool_find_and_retain(self.h, _p(t), t.size)
        return None if b < 0 else b

    def publish(self, block, prefix):
        t = self._toks(prefix)
        library().nvbh_pool_publish(self.h, block, _p(t), t.size)

    def available(self):
        return library().nvbh_pool_available(self.h)

    def in_use(self):
        return library().nvbh_pool_in_use(self.h)

    def references(self, block):
        return library().nvbh_pool_references(self.h, block)

    def cached_keys(self):
        return library().nvbh_pool_cached_keys(self.h)

    def clear_cache(self):
        library().nvbh_pool_clear_cache(self.h)

    def force_hash_entry(self, prefix, block):
        t = self._toks(prefix)
        library().nvbh_pool_force_hash_entry(self.h, _p(t), t.size, block)


@dataclass
class Segment:
    tokens: list
    blocks: list
    start: int
    end: int
    sample: bool = False
    request_id: int = 0
    generated: int = 0
    temperature: float = 0.0


def make_batch(segments, block_size, seed, is_decode=False) -> Batch:
    """Flattens segments into a Batch (src/runtime.rs:728-777)."""
    keep = []
    cs = (NvbhSegment * max(1, len(segments)))()
    rows = 0
    stride = max([len(s.blocks) for s in segments], default=0)
    for i, s in enumerate(segments):
        t, b = _arr(s.tokens, np.uint32), _arr(s.blocks, np.int32)
        keep += [t, b]
        cs[i] = NvbhSegment(_p(t), t.size, _p(b), b.size, s.start, s.end, int(s.sample), s.request_id, s.generated,
                            s.temperature)
        rows += max(0, s.end - s.start)
    n = len(segments)
    out = dict(token_ids=np.zeros(max(rows, 1), np.int32), positions=np.zeros(max(rows, 1), np.int32),
               sequence_ids=np.zeros(max(rows, 1), np.int32), slot_mapping=np.zeros(max(rows, 1), np.int32),
               block_tables=np.zeros(max(n * stride, 1), np.int32), last=np.zeros(max(n, 1), np.int32),
               temps=np.zeros(max(n, 1), np.float32), seeds=np.zeros(max(n, 1), np.uint64))
    co = NvbhBatchOut(_p(out["token_ids"]), _p(out["positions"]), _p(out["sequence_ids"]), _p(out["slot_mapping"]),
                      rows, _p(out["block_tables"]), n * stride, _p(out["last"]), _p(out["temps"]), _p(out["seeds"]),
                      n, 0, 0, 0)
    _check(library().nvbh_make_batch(cs, n, block_size, seed, ctypes.byref(co)))
    r, k = co.rows, co.samples
    return Batch(token_ids=out["token_ids"][:r].tolist(), positions=out["positions"][:r].tolist(),
                 sequence_ids=out["sequence_ids"][:r].tolist(), slot_mapping=out["slot_mapping"][:r].tolist(),
                 block_tables=out["block_tables"][:n * co.table_stride].tolist(), table_stride=co.table_stride,
                 last_token_indices=out["last"][:k].tolist(), temperatures=out["temps"][:k].tolist(),
                 seeds=[int(x) for x in out["seeds"][:k]], is_decode=is_decode)


def sampling_seed(base, request_id, generated):
    return int(library().nvbh_sampling_seed(base, request_id, generated))
