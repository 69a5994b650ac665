"""Continuous-batching engine (libnvb_host.so, nvbe_engine_*) from Python.

Mirrors the reference's runtime API (src/runtime.rs): `SchedulerConfig`,
`Request`, `LlmEngine.generate(requests, seed)` returning outputs in request
order plus `RunStats`. The scheduler itself is C++ (engine.cpp); a runner is
either this package's GPU model (`model.Qwen3Model`, called C to C with no
Python in the step loop) or any Python object with
`run(batch: Batch) -> list[int]` (called through a ctypes callback; used by
the CPU tests, like the reference's mock runners in src/runtime/tests.rs).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import host as _host

c_size = ctypes.c_size_t
P = ctypes.c_void_p


class NvbeSchedulerConfig(ctypes.Structure):
    _fields_ = [("block_size", c_size), ("num_blocks", c_size), ("max_sequences", c_size),
                ("max_model_len", c_size), ("max_batch_tokens", c_size), ("prefix_caching", ctypes.c_int),
                ("eos_token_id", ctypes.c_int64), ("mixed_batches", ctypes.c_int)]


class NvbeRequest(ctypes.Structure):
    _fields_ = [("id", ctypes.c_uint64), ("prompt_token_ids", P), ("prompt_len", c_size), ("max_tokens", c_size),
                ("temperature", ctypes.c_float), ("ignore_eos", ctypes.c_int)]


class NvbeRequestOutput(ctypes.Structure):
    _fields_ = [("token_ids", P), ("num_tokens", c_size), ("prompt_tokens", c_size), ("cached_tokens", c_size),
                ("ttft_ms", ctypes.c_double), ("latency_ms", ctypes.c_double), ("inter_token_latencies_ms", P),
                ("num_gaps", c_size), ("finish_reason", ctypes.c_int)]


STAT_FIELDS = [("elapsed_seconds", ctypes.c_double), ("input_tokens", c_size), ("output_tokens", c_size),
               ("output_tokens_per_second", ctypes.c_double), ("total_requests", c_size),
               ("cached_tokens", c_size), ("cache_hits", c_size), ("prefill_tokens", c_size),
               ("decode_tokens", c_size), ("prefill_steps", c_size), ("decode_steps", c_size),
               ("prefill_seconds", ctypes.c_double), ("decode_seconds", ctypes.c_double),
               ("preemptions", c_size), ("peak_kv_blocks", c_size), ("mean_ttft_ms", ctypes.c_double),
               ("mean_latency_ms", ctypes.c_double), ("mean_inter_token_latency_ms", ctypes.c_double),
               ("mixed_steps", c_size), ("mixed_seconds", ctypes.c_double)]


class NvbeRunStats(ctypes.Structure):
    _fields_ = STAT_FIELDS


RUN_FN = ctypes.CFUNCTYPE(ctypes.c_int, P, ctypes.POINTER(_host.NvbhBatch), ctypes.POINTER(ctypes.c_uint32))
SYNC_FN = ctypes.CFUNCTYPE(ctypes.c_int, P)

_declared = False


def _lib():
    global _declared
    L = _host.library()
    if not _declared:
        L.nvbe_engine_last_error.restype = ctypes.c_char_p
        L.nvbe_scheduler_config_validate.argtypes = [ctypes.POINTER(NvbeSchedulerConfig)]
        L.nvbe_engine_create.argtypes = [ctypes.POINTER(NvbeSchedulerConfig), P, P, P, ctypes.POINTER(P)]
        L.nvbe_engine_destroy.argtypes = [P]
        L.nvbe_engine_destroy.restype = None
        L.nvbe_engine_generate.argtypes = [P, ctypes.POINTER(NvbeRequest), c_size, ctypes.c_uint64,
                                           ctypes.POINTER(NvbeRequestOutput), ctypes.POINTER(NvbeRunStats)]
        L.nvbe_engine_clear_prefix_cache.argtypes = [P]
        L.nvbe_engine_blocks_in_use.argtypes = [P]
        L.nvbe_engine_blocks_in_use.restype = c_size
        L.nvbe_engine_cached_keys.argtypes = [P]
        L.nvbe_engine_cached_keys.restype = c_size
        _declared = True
    return L


class EngineError(RuntimeError):
    pass


@dataclass
class SchedulerConfig:
    """SchedulerConfig (src/runtime.rs:73-97), with the reference's defaults."""
    block_size: int = 256
    num_blocks: int = 128
    max_sequences: int = 32
    max_model_len: int = 4096
    max_batch_tokens: int = 1024
    prefix_caching: bool = True
    eos_token_id: int | None = None
    # This build's addition: decode rows and prefill chunks in one forward
    # (False keeps the reference's separate forwards).
    mixed_batches: bool = False

    def to_c(self):
        return NvbeSchedulerConfig(self.block_size, self.num_blocks, self.max_sequences, self.max_model_len,
                                   self.max_batch_tokens, int(self.prefix_caching),
                                   -1 if self.eos_token_id is None else int(self.eos_token_id),
                                   int(self.mixed_batches))

    def validate(self):
        c = self.to_c()
        if _lib().nvbe_scheduler_config_validate(ctypes.byref(c)):
            raise EngineError(_lib().nvbe_engine_last_error().decode())


@dataclass
class Request:
    """Request (src/runtime.rs:51-71)."""
    id: int
    prompt_token_ids: list
    max_tokens: int = 32
    temperature: float = 0.0
    ignore_eos: bool = False


@dataclass
class RequestOutput:
    id: int
    token_ids: list
    prompt_tokens: int
    cached_tokens: int
    ttft_ms: float
    latency_ms: float
    inter_token_latencies_ms: list
    finish_reason: str


@dataclass
class RunOutput:
    outputs: list
    stats: dict = field(default_factory=dict)


@dataclass
class Batch:
    """A forward pass as a Python runner sees it (the reference's Batch,
    src/runtime.rs:15-39), copied out of the engine's buffers."""
    token_ids: np.ndarray
    positions: np.ndarray
    sequence_ids: np.ndarray
    slot_mapping: np.ndarray
    block_tables: np.ndarray
    table_stride: int
    last_token_indices: np.ndarray
    temperatures: np.ndarray
    seeds: np.ndarray
    is_decode: bool

    def sequence_count(self):
        return len(self.block_tables) // self.table_stride if self.table_stride else 0

    @staticmethod
    def from_c(b):
        def arr(ptr, n, ctype, dtype):
            if n == 0:
                return np.zeros(0, dtype=dtype)
            return np.ctypeslib.as_array(ctypes.cast(ptr, ctypes.POINTER(ctype)), shape=(n,)).astype(dtype)

        return Batch(arr(b.token_ids, b.rows, ctypes.c_int32, np.int32),
                     arr(b.positions, b.rows, ctypes.c_int32, np.int32),
                     arr(b.sequence_ids, b.rows, ctypes.c_int32, np.int32),
                     arr(b.slot_mapping, b.rows, ctypes.c_int32, np.int32),
                     arr(b.block_tables, b.block_tables_len, ctypes.c_int32, np.int32), int(b.table_stride),
                     arr(b.last_token_indices, b.samples, ctypes.c_int32, np.int32),
                     arr(b.temperatures, b.samples, ctypes.c_float, np.float32),
                     arr(b.seeds, b.samples, ctypes.c_uint64, np.uint64), bool(b.is_decode))


class LlmEngine:
    """LlmEngine (src/runtime.rs:360-409) over the C++ scheduler."""

    def __init__(self, config: SchedulerConfig, runner):
        self.config = config
        self.runner = runner
        c = config.to_c()
        handle = P()
        if hasattr(runner, "c_run_fn"):
            run_fn, sync_fn, ctx = runner.c_run_fn(), runner.c_sync_fn(), runner.c_handle()
            self._callbacks = None
        else:
            self._error = None

            def run(_ctx, batch_ptr, sampled_ptr):
                try:
                    batch = Batch.from_c(batch_ptr.contents)
                    out = runner.run(batch)
                    if len(out) != len(batch.last_token_indices):
                        raise EngineError(f"runner returned {len(out)} samples for {len(batch.last_token_indices)}")
                    for i, t in enumerate(out):
                        sampled_ptr[i] = int(t)
                    return 0
                except Exception as e:  # reported by generate()
                    self._error = e
                    return 1

            def sync(_ctx):
                s = getattr(runner, "synchronize", None)
                try:
                    if s:
                        s()
                    return 0
                except Exception as e:
                    self._error = e
                    return 1

            self._callbacks = (RUN_FN(run), SYNC_FN(sync))
            run_fn = ctypes.cast(self._callbacks[0], P)
            sync_fn = ctypes.cast(self._callbacks[1], P)
            ctx = P(0)
        L = _lib()
        if L.nvbe_engine_create(ctypes.byref(c), run_fn, sync_fn, ctx, ctypes.byref(handle)):
            raise EngineError(L.nvbe_engine_last_error().decode())
        self._handle = handle

    def close(self):
        if getattr(self, "_handle", None):
            _lib().nvbe_engine_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def blocks_in_use(self):
        return _lib().nvbe_engine_blocks_in_use(self._handle)

    def cached_keys(self):
        return _lib().nvbe_engine_cached_keys(self._handle)

    def clear_prefix_cache(self):
        if _lib().nvbe_engine_clear_prefix_cache(self._handle):
            raise EngineError(_lib().nvbe_engine_last_error().decode())

    def generate(self, requests, seed: int) -> RunOutput:
        n = len(requests)
        reqs = (NvbeRequest * max(n, 1))()
        outs = (NvbeRequestOutput * max(n, 1))()
        keep = []
        for i, r in enumerate(requests):
            if any(int(t) < 0 or int(t) >= 2**32 for t in r.prompt_token_ids):
                raise EngineError("token IDs must fit in u32")
            prompt = np.ascontiguousarray(np.asarray(r.prompt_token_ids, dtype=np.uint64).astype(np.uint32))
            if r.max_tokens < 0:
                raise EngineError("max_tokens must be nonnegative")
            # generate() rejects a request whose max_tokens exceeds
            # max_model_len before anything is written to its buffer
            cap = int(r.max_tokens) if 0 < r.max_tokens <= self.config.max_model_len else 1
            tokens = np.zeros(cap, dtype=np.uint32)
            gaps = np.zeros(len(tokens), dtype=np.float64)
            keep += [prompt, tokens, gaps]
            reqs[i] = NvbeRequest(int(r.id), prompt.ctypes.data if len(prompt) else None, len(prompt),
                                  int(r.max_tokens), float(r.temperature), int(r.ignore_eos))
            outs[i] = NvbeRequestOutput(tokens.ctypes.data, 0, 0, 0, 0.0, 0.0, gaps.ctypes.data, 0, 0)
        stats = NvbeRunStats()
        L = _lib()
        rc = L.nvbe_engine_generate(self._handle, reqs, n, ctypes.c_uint64(seed), outs, ctypes.byref(stats))
        if rc:
            msg = L.nvbe_engine_last_error().decode()
            err = getattr(self, "_error", None)
            if err is not None:
                self._error = None
                raise EngineError(f"{msg}: {err!r}") from err
            detail = self.runner.last_error() if hasattr(self.runner, "last_error") else ""
            raise EngineError(f"{msg} {detail}".strip())
        results = []
        for i, r in enumerate(requests):
            o = outs[i]
            tokens = keep[3 * i + 1][:o.num_tokens].tolist()
            gaps = keep[3 * i + 2][:o.num_gaps].tolist()
            results.append(RequestOutput(r.id, tokens, o.prompt_tokens, o.cached_tokens, o.ttft_ms, o.latency_ms,
                                         gaps, "eos" if o.finish_reason == 1 else "length"))
        return RunOutput(results, {name: getattr(stats, name) for name, _ in STAT_FIELDS})


def sampling_seed(base, request_id, generated):
    """Per-request, per-step seed (src/runtime.rs:782-790)."""
    L = _host.library()
    L.nvbh_sampling_seed.restype = ctypes.c_uint64
    L.nvbh_sampling_seed.argtypes = [ctypes.c_uint64] * 3
    return int(L.nvbh_sampling_seed(base, request_id, generated))
