"""The reference engine's model runner, for parity tests only.

A Python restatement of the reference's QwenModel::forward and ::run with
the native attention backend (src/model.rs:635-818, 924-1003) that calls the
reference's own kernels through their C ABI (kernels/kernels.cu, built from
its sources into oracle/_ref/libref_native.so): nv_embedding, nv_rms,
nv_add_rms, nv_gemm (cuBLAS), nv_qkv_rope_cached, nv_attention, nv_silu,
nv_gather, nv_sample_parallel. It plugs into the engine's scheduler like any
runner (`run(batch) -> sampled ids`), so both runners see the same batches.
It owns its own K/V caches and workspace; the weights are shared, read-only.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float


def declare(L):
    L.nv_embedding.argtypes = [P] * 4 + [I] * 3
    L.nv_rms.argtypes = [P] * 4 + [I, I, F]
    L.nv_add_rms.argtypes = [P] * 5 + [I, I, F]
    L.nv_gemm.argtypes = [P] * 4 + [I] * 3
    L.nv_qkv_rope_cached.argtypes = [P] * 9 + [I] * 6 + [F, P, I]
    L.nv_rope_cache.argtypes = [P, P, I, I, F]
    L.nv_attention.argtypes = [P] * 8 + [I] * 9
    L.nv_silu.argtypes = [P] * 3 + [I, I]
    L.nv_gather.argtypes = [P] * 4 + [I] * 3
    L.nv_sample_parallel.argtypes = [P] * 7 + [I, I]
    L.nv_sample.argtypes = [P] * 5 + [I, I]


def _p(t):
    return P(t.data_ptr())


class RefRunner:
    """QwenModel on the reference's kernels, with its native attention
    backend (nv_attention) or, given `flash` (oracle/_ref/libref_flash.so),
    its FA2 backend (nvr_flash_fwd with flash_metadata, src/model.rs:234-267,
    698-726, and per-batch decode splits fixed by max_model_len,
    src/model.rs:414-439, 947-949)."""

    def __init__(self, ref_native, config, options, weights, flash=None, nvb=None):
        self.ref = ref_native
        self.flash = flash
        self.nvb = nvb  # this library's package: its attention in the reference forward (a diagnostic hybrid)
        declare(ref_native.L)
        self.c, self.o, self.w = config, options, weights
        c, o = config, options
        dev = torch.device("cuda", o.device)
        self.table_stride = -(-o.max_model_len // o.block_size)
        T, S, H, D = o.max_batch_tokens, o.max_sequences, c.hidden_size, c.head_dim
        qh, kvh, Iz = c.num_attention_heads, c.num_key_value_heads, c.intermediate_size
        bf = dict(dtype=torch.bfloat16, device=dev)
        z = lambda *s, **kw: torch.zeros(*s, **{**bf, **kw})  # noqa: E731
        self.residual, self.hidden, self.normed = z(T, H), z(T, H), z(T, H)
        self.qkv, self.query, self.attention = z(T, (qh + 2 * kvh) * D), z(T, qh * D), z(T, qh * D)
        self.gate_up, self.activated = z(T, 2 * Iz), z(T, Iz)
        self.gathered, self.logits = z(S, H), z(S, c.vocab_size)
        parts = -(-c.vocab_size // 2048)
        self.part_scores = torch.zeros(S * parts, dtype=torch.float32, device=dev)
        self.part_ids = torch.zeros(S * parts, dtype=torch.int32, device=dev)
        self.samples = torch.zeros(S, dtype=torch.int32, device=dev)
        self.rope = torch.zeros(o.max_model_len, D, dtype=torch.float32, device=dev)
        cache = (o.num_blocks, o.block_size, kvh, D)
        self.k = [z(*cache) for _ in range(c.num_hidden_layers)]
        self.v = [z(*cache) for _ in range(c.num_hidden_layers)]
        if nvb is not None:
            import ctypes as C

            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            self.nsplits = [1] + [max(1, nvb.num_splits(b, qh, kvh, o.max_model_len, sms)) for b in range(1, S + 1)]
            ms = max(self.nsplits)
            self.n_la = torch.zeros(ms * S * qh, dtype=torch.float32, device=dev)
            self.n_oa = torch.zeros(ms * S * qh * D, dtype=torch.float32, device=dev)
            sp = P()
            ref_native.L.nv_stream(ref_native.ctx, C.byref(sp))
            self.stream = sp
        if flash is not None:
            import ctypes as C

            flash.nvr_flash_fwd.argtypes = [P] * 8 + [I] * 9 + [P] * 3
            flash.nvr_flash_num_splits.argtypes = [I] * 5
            flash.nvr_flash_last_error.restype = C.c_char_p
            sms = torch.cuda.get_device_properties(dev).multi_processor_count
            self.splits = [1] + [flash.nvr_flash_num_splits(b, qh, kvh, o.max_model_len, sms) for b in range(1, S + 1)]
            ms = max(self.splits)
            self.lse = torch.zeros(S * qh * T, dtype=torch.float32, device=dev)
            self.lse_accum = torch.zeros(ms * S * qh, dtype=torch.float32, device=dev)
            self.out_accum = torch.zeros(ms * S * qh * D, dtype=torch.float32, device=dev)
            sp = P()
            ref_native.L.nv_stream(ref_native.ctx, C.byref(sp))
            self.stream = sp
        torch.cuda.synchronize()
        self.call("nv_rope_cache", self.rope, o.max_model_len, D, c.rope_theta)
        self.ref.sync()
        self.dev = dev
        self.last_samples = 0

    def call(self, name, *args):
        conv = [_p(a) if isinstance(a, torch.Tensor) else a for a in args]
        self.ref._check(getattr(self.ref.L, name)(self.ref.ctx, *conv))

    def forward(self, rows, sequences, samples, m):
        c, o, w = self.c, self.o, self.w
        H, D, qh, kvh, Iz = c.hidden_size, c.head_dim, c.num_attention_heads, c.num_key_value_heads, \
            c.intermediate_size
        q_size, qkv_size, eps = qh * D, (qh + 2 * kvh) * D, c.rms_norm_eps
        self.call("nv_embedding", m["tokens"], w["embedding"], self.residual, rows, H, c.vocab_size)
        for l, lw in enumerate(w["layers"]):
            if l == 0:
                self.call("nv_rms", self.residual, lw["input_norm"], self.normed, rows, H, eps)
            else:
                self.call("nv_add_rms", self.hidden, self.residual, lw["input_norm"], self.normed, rows, H, eps)
            self.call("nv_gemm", self.normed, lw["qkv"], self.qkv, rows, qkv_size, H)
            self.call("nv_qkv_rope_cached", self.qkv, lw["q_norm"], lw["k_norm"], m["positions"], m["slots"],
                      self.query, self.k[l], self.v[l], rows, qh, kvh, D, o.block_size, o.num_blocks, eps, self.rope,
                      o.max_model_len)
            if self.nvb is not None:
                splits = self.nsplits[sequences] if m["max_q"] == 1 else 1
                lib = self.nvb.library()
                rc = lib.nvb_paged_fwd_ex(self.stream, _p(self.query), _p(self.k[l]), _p(self.v[l]),
                                          _p(self.attention), _p(m["cu_q"]), _p(m["kv_lens"]), _p(m["tables"]),
                                          sequences, rows, m["max_q"], m["max_k"], qh, kvh, o.block_size,
                                          self.table_stride, splits, None, _p(self.n_la), _p(self.n_oa),
                                          o.num_blocks)
                if rc:
                    raise RuntimeError(lib.nvb_last_error().decode())
            elif self.flash is None:
                self.call("nv_attention", self.query, self.k[l], self.v[l], m["positions"], m["seqs"], m["tables"],
                          self.attention, rows, qh, kvh, D, o.block_size, o.num_blocks, self.table_stride, sequences,
                          o.max_model_len)
            else:
                splits = self.splits[sequences] if m["max_q"] == 1 else 1
                rc = self.flash.nvr_flash_fwd(self.stream, _p(self.query), _p(self.k[l]), _p(self.v[l]),
                                              _p(self.attention), _p(m["cu_q"]), _p(m["kv_lens"]), _p(m["tables"]),
                                              sequences, rows, m["max_q"], m["max_k"], qh, kvh, o.block_size,
                                              self.table_stride, splits, _p(self.lse), _p(self.lse_accum),
                                              _p(self.out_accum))
                if rc:
                    raise RuntimeError(self.flash.nvr_flash_last_error().decode())
            self.call("nv_gemm", self.attention, lw["o_proj"], self.hidden, rows, H, q_size)
            self.call("nv_add_rms", self.hidden, self.residual, lw["post_norm"], self.normed, rows, H, eps)
            self.call("nv_gemm", self.normed, lw["gate_up"], self.gate_up, rows, 2 * Iz, H)
            self.call("nv_silu", self.gate_up, self.activated, rows, Iz)
            self.call("nv_gemm", self.activated, lw["down"], self.hidden, rows, H, Iz)
        if samples:
            self.call("nv_add_rms", self.hidden, self.residual, w["final_norm"], self.normed, rows, H, eps)
            self.call("nv_gather", self.normed, m["last"], self.gathered, samples, H, rows)
            lm = w["lm_head"] if w.get("lm_head") is not None else w["embedding"]
            self.call("nv_gemm", self.gathered, lm, self.logits, samples, c.vocab_size, H)
            self.call("nv_sample_parallel", self.logits, m["temps"], m["seeds"], self.samples, self.part_scores,
                      self.part_ids, samples, c.vocab_size)

    def run(self, batch):
        """ModelRunner::run (src/model.rs:924-1003), eager, native backend."""
        rows = len(batch.token_ids)
        sequences = batch.sequence_count()
        samples = len(batch.last_token_indices)
        tables = np.full((sequences, self.table_stride), -1, dtype=np.int32)
        bt = np.asarray(batch.block_tables, dtype=np.int32).reshape(sequences, batch.table_stride)
        tables[:, :batch.table_stride] = bt
        to = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a).astype(dt)).to(self.dev)  # noqa: E731
        m = {"tokens": to(batch.token_ids, np.int32), "positions": to(batch.positions, np.int32),
             "seqs": to(batch.sequence_ids, np.int32), "slots": to(batch.slot_mapping, np.int32),
             "tables": to(tables, np.int32), "last": to(batch.last_token_indices, np.int32),
             "temps": to(batch.temperatures, np.float32),
             "seeds": to(np.asarray(batch.seeds, dtype=np.uint64).view(np.int64), np.int64)}
        if self.flash is not None or self.nvb is not None:
            # flash_metadata (src/model.rs:234-267): consecutive query groups per sequence
            seq = np.asarray(batch.sequence_ids)
            pos = np.asarray(batch.positions)
            counts = np.bincount(seq, minlength=sequences)
            cu = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
            lens = np.array([pos[cu[b + 1] - 1] + 1 for b in range(sequences)], dtype=np.int32)
            m["cu_q"], m["kv_lens"] = to(cu, np.int32), to(lens, np.int32)
            m["max_q"] = int(counts.max())
            m["max_k"] = self.o.max_model_len if m["max_q"] == 1 else int(lens.max())
        torch.cuda.synchronize()  # the upload is complete before the reference stream reads it
        self.forward(rows, sequences, samples, m)
        self.ref.sync()
        self.last_samples = samples
        return self.samples[:samples].cpu().tolist() if samples else []

    def last_logits(self):
        return self.logits[: self.last_samples].cpu()
