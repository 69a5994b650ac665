"""Qwen3 model runner on one GPU (libnvb_model.so, nvbe_model_*) from Python.

`Qwen3Model` owns the runner: paged K/V caches, workspace, its CUDA stream
and cuBLAS handle, decode CUDA graphs. The weights are caller-owned torch
tensors (the reference loads safetensors; there is no checkpoint here, so
`random_weights` draws a seeded random initialisation of the architecture).
An `engine.LlmEngine` drives it C to C: the scheduler calls nvbe_model_run
directly, with no Python in the step loop.

The per-layer kernels are exposed too (`layer_*`): each replaces one of the
reference's nv_* entry points (kernels/kernels.cu:470-500) with a stream.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

from . import host as _host  # noqa: F401  (loads libnvb_host.so first)

P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
_lib = None


class NvbeModelConfig(ctypes.Structure):
    _fields_ = [("hidden_size", I), ("intermediate_size", I), ("num_hidden_layers", I),
                ("num_attention_heads", I), ("num_key_value_heads", I), ("head_dim", I), ("vocab_size", I),
                ("rms_norm_eps", F), ("rope_theta", F), ("tie_word_embeddings", I)]


class NvbeModelOptions(ctypes.Structure):
    _fields_ = [("device", I), ("block_size", I), ("num_blocks", I), ("max_batch_tokens", I),
                ("max_sequences", I), ("max_model_len", I), ("cuda_graphs", I), ("tc_gemms", I)]


class NvbeModelWeights(ctypes.Structure):
    _fields_ = [("embedding", P), ("final_norm", P), ("lm_head", P)] + [
        (n, P) for n in ("input_norm", "qkv", "q_norm", "k_norm", "o_proj", "post_norm", "gate_up", "down")]


LAYER_FIELDS = ("input_norm", "qkv", "q_norm", "k_norm", "o_proj", "post_norm", "gate_up", "down")


def library():
    """Loads libnvb_model.so (and, through it, libnvb.so / libnvb_host.so)."""
    global _lib
    if _lib is None:
        from . import LIB_DIR, library as attention_library

        attention_library()
        path = LIB_DIR / "libnvb_model.so"
        if not path.exists():
            raise RuntimeError(f"{path} is missing: run __graft_entry__.build() first")
        L = ctypes.CDLL(str(path))
        L.nvbe_model_last_error.restype = ctypes.c_char_p
        L.nvbe_model_create.argtypes = [ctypes.POINTER(NvbeModelConfig), ctypes.POINTER(NvbeModelOptions),
                                        ctypes.POINTER(NvbeModelWeights), ctypes.POINTER(P)]
        L.nvbe_model_destroy.argtypes = [P]
        L.nvbe_model_destroy.restype = None
        L.nvbe_model_sync.argtypes = [P]
        L.nvbe_model_last_logits.argtypes = [P, P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]
        L.nvbe_model_kv_cache.argtypes = [P, I, ctypes.POINTER(P), ctypes.POINTER(P)]
        L.nvbe_model_stream.argtypes = [P]
        L.nvbe_model_stream.restype = P
        L.nvbe_model_graph_count.argtypes = [P]
        L.nvbe_model_graph_count.restype = ctypes.c_size_t
        L.nvbe_layer_embedding.argtypes = [P] * 4 + [I] * 3
        L.nvbe_layer_rms.argtypes = [P] * 4 + [I, I, F]
        L.nvbe_layer_add_rms.argtypes = [P] * 5 + [I, I, F]
        L.nvbe_layer_silu_mul.argtypes = [P] * 3 + [I, I]
        L.nvbe_layer_gather.argtypes = [P] * 4 + [I] * 3
        L.nvbe_layer_gemm.argtypes = [P, P, P, P, I, I, I, I, P, ctypes.c_size_t]
        L.nvbe_gemm_workspace_bytes.argtypes = [I, I, I, I]
        L.nvbe_gemm_workspace_bytes.restype = ctypes.c_size_t
        L.nvbe_gemm_device_error.argtypes = []
        L.nvbe_gemm_sample_tiles.argtypes = [I]
        L.nvbe_layer_gemm_sample.argtypes = [P, P, P, P, I, I, I, P, P, P, P, P]
        L.nvbe_sample_partitions.argtypes = [I]
        L.nvbe_layer_sample.argtypes = [P] * 7 + [I, I]
        _lib = L
    return _lib


class ModelError(RuntimeError):
    pass


def _check(rc):
    if rc:
        raise ModelError(f"libnvb_model: {library().nvbe_model_last_error().decode(errors='replace')} (status {rc})")


@dataclass
class Qwen3Config:
    """The config.json fields the forward uses (src/model.rs:19-49);
    defaults are Qwen3-0.6B's."""
    hidden_size: int = 1024
    intermediate_size: int = 3072
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    vocab_size: int = 151936
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    tie_word_embeddings: bool = True

    def to_c(self):
        return NvbeModelConfig(self.hidden_size, self.intermediate_size, self.num_hidden_layers,
                               self.num_attention_heads, self.num_key_value_heads, self.head_dim, self.vocab_size,
                               self.rms_norm_eps, self.rope_theta, int(self.tie_word_embeddings))


@dataclass
class ModelOptions:
    """ModelOptions (src/model.rs:151-181)."""
    device: int = 0
    block_size: int = 256
    num_blocks: int = 128
    max_batch_tokens: int = 1024
    max_sequences: int = 32
    max_model_len: int = 4096
    cuda_graphs: bool = True
    tc_gemms: bool = True  # tcgen05 GEMMs for forwards of <= 256 rows (else cuBLAS)

    def to_c(self):
        return NvbeModelOptions(self.device, self.block_size, self.num_blocks, self.max_batch_tokens,
                                self.max_sequences, self.max_model_len, int(self.cuda_graphs), int(self.tc_gemms))


def random_weights(config: Qwen3Config, seed=0, device="cuda", std=0.02):
    """Seeded random initialisation of the architecture in the checkpoint's
    row-major [out, in] BF16 layout: embedding and projection weights
    N(0, std), RMSNorm weights N(1, std). Per layer `qkv` stacks q_proj,
    k_proj and v_proj rows and `gate_up` stacks gate_proj and up_proj rows,
    as the reference uploads them (src/model.rs:455-504)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    c = config
    H, D, Iz = c.hidden_size, c.head_dim, c.intermediate_size
    qkv_rows = (c.num_attention_heads + 2 * c.num_key_value_heads) * D

    def normal(*shape, mean=0.0):
        t = torch.empty(*shape, dtype=torch.float32, device=device)
        t.normal_(mean, std, generator=g)
        return t.to(torch.bfloat16)

    w = {"embedding": normal(c.vocab_size, H), "final_norm": normal(H, mean=1.0),
         "lm_head": None if c.tie_word_embeddings else normal(c.vocab_size, H)}
    layers = []
    for _ in range(c.num_hidden_layers):
        layers.append({"input_norm": normal(H, mean=1.0), "qkv": normal(qkv_rows, H), "q_norm": normal(D, mean=1.0),
                       "k_norm": normal(D, mean=1.0), "o_proj": normal(H, c.num_attention_heads * D),
                       "post_norm": normal(H, mean=1.0), "gate_up": normal(2 * Iz, H), "down": normal(H, Iz)})
    w["layers"] = layers
    return w


class _DeviceArray:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3, "strides": None}


class Qwen3Model:
    """QwenModel (src/model.rs:361-1003) on this library's kernels."""

    def __init__(self, config: Qwen3Config, options: ModelOptions, weights):
        import torch

        L = library()
        self.config, self.options, self.weights = config, options, weights
        # the runner has its own stream: the weights must be complete first
        torch.cuda.synchronize(options.device)
        layers = weights["layers"]
        n = config.num_hidden_layers
        if len(layers) != n:
            raise ModelError(f"{len(layers)} layers of weights for {n} layers")
        self._arrays = {f: (P * n)(*[layers[i][f].data_ptr() for i in range(n)]) for f in LAYER_FIELDS}
        lm = weights.get("lm_head")
        cw = NvbeModelWeights(weights["embedding"].data_ptr(), weights["final_norm"].data_ptr(),
                              lm.data_ptr() if lm is not None else None,
                              *[ctypes.cast(self._arrays[f], P) for f in LAYER_FIELDS])
        self._cfg, self._opt = config.to_c(), options.to_c()
        handle = P()
        _check(L.nvbe_model_create(ctypes.byref(self._cfg), ctypes.byref(self._opt), ctypes.byref(cw),
                                   ctypes.byref(handle)))
        self._handle = handle

    # the NvbeRunFn / NvbeSyncFn pair an engine calls directly
    def c_run_fn(self):
        return ctypes.cast(library().nvbe_model_run, P)

    def c_sync_fn(self):
        return ctypes.cast(library().nvbe_model_sync, P)

    def c_handle(self):
        return self._handle

    def last_error(self):
        return library().nvbe_model_last_error().decode(errors="replace")

    def synchronize(self):
        _check(library().nvbe_model_sync(self._handle))

    def graph_count(self):
        return library().nvbe_model_graph_count(self._handle)

    def stream_ptr(self):
        return library().nvbe_model_stream(self._handle)

    def last_logits(self):
        """BF16 logits [samples, vocab] of the latest run, as a CPU tensor."""
        import torch

        n = ctypes.c_size_t()
        cap = self.options.max_sequences * self.config.vocab_size
        out = torch.empty(cap, dtype=torch.int16)
        _check(library().nvbe_model_last_logits(self._handle, P(out.data_ptr()), cap, ctypes.byref(n)))
        return out[: n.value * self.config.vocab_size].view(torch.bfloat16).view(n.value, self.config.vocab_size)

    def kv_cache(self, layer):
        """Layer `layer`'s K and V caches as torch views
        [num_blocks, block_size, kv_heads, head_dim] BF16."""
        import torch

        k, v = P(), P()
        _check(library().nvbe_model_kv_cache(self._handle, layer, ctypes.byref(k), ctypes.byref(v)))
        o, c = self.options, self.config
        shape = (o.num_blocks, o.block_size, c.num_key_value_heads, c.head_dim)
        dev = torch.device("cuda", o.device)
        return tuple(torch.as_tensor(_DeviceArray(p.value, shape, "<i2"), device=dev).view(torch.bfloat16)
                     for p in (k, v))

    def close(self):
        if getattr(self, "_handle", None):
            library().nvbe_model_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------- layer kernels
def _s(stream):
    import torch

    return P((stream or torch.cuda.current_stream()).cuda_stream)


def _p(t):
    return P(t.data_ptr())


def layer_embedding(tokens, weight, out, stream=None):
    rows, hidden = out.shape
    _check(library().nvbe_layer_embedding(_s(stream), _p(tokens), _p(weight), _p(out), rows, hidden, weight.shape[0]))


def layer_rms(x, weight, out, eps, stream=None):
    rows, hidden = x.shape
    _check(library().nvbe_layer_rms(_s(stream), _p(x), _p(weight), _p(out), rows, hidden, eps))


def layer_add_rms(x, residual, weight, out, eps, stream=None):
    rows, hidden = x.shape
    _check(library().nvbe_layer_add_rms(_s(stream), _p(x), _p(residual), _p(weight), _p(out), rows, hidden, eps))


def layer_silu_mul(packed, out, stream=None):
    rows, inter = out.shape
    _check(library().nvbe_layer_silu_mul(_s(stream), _p(packed), _p(out), rows, inter))


def layer_gather(x, indices, out, stream=None):
    rows, hidden = out.shape
    _check(library().nvbe_layer_gather(_s(stream), _p(x), _p(indices), _p(out), rows, hidden, x.shape[0]))


def gemm_workspace_bytes(m, n, k, silu=False):
    return library().nvbe_gemm_workspace_bytes(m, n, k, int(silu))


def layer_gemm(x, w, y, silu=False, stream=None, workspace=None):
    """nvbe_layer_gemm: y = x w^T ([M, K] x [N, K] -> [M, N]) on the tcgen05
    decode GEMM, or y[M, N / 2] = silu(gate) * up with silu=True. `workspace`
    (a CUDA uint8 tensor of gemm_workspace_bytes) is allocated per call when
    not given."""
    import torch

    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] != K or x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or y.dtype != torch.bfloat16:
        raise ValueError("x [M, K], w [N, K] and y must be BF16 with matching K")
    if tuple(y.shape) != (M, N // 2 if silu else N) or not (x.is_contiguous() and w.is_contiguous() and y.is_contiguous()):
        raise ValueError("y must be a contiguous [M, N] (or [M, N / 2] with silu) tensor")
    nbytes = library().nvbe_gemm_workspace_bytes(M, N, K, int(silu))
    ws = workspace if workspace is not None else torch.empty(max(16, nbytes), dtype=torch.uint8, device=x.device)
    _check(library().nvbe_layer_gemm(_s(stream), _p(x), _p(w), _p(y), M, N, K, int(silu), _p(ws), ws.numel()))


def layer_gemm_sample(x, w, logits, temperatures, seeds, out, stream=None):
    """nvbe_layer_gemm_sample: logits = x w^T and out = the Gumbel-max samples
    of those logits (the reference sampler's stream), in one fused launch
    plus the per-tile fold."""
    import torch

    M, K = x.shape
    N = w.shape[0]
    if tuple(logits.shape) != (M, N) or logits.dtype != torch.bfloat16 or out.shape[0] != M:
        raise ValueError("logits must be [M, N] BF16 and out [M] int32")
    tiles = library().nvbe_gemm_sample_tiles(N)
    ps = torch.empty(M * tiles, dtype=torch.float32, device=x.device)
    pi = torch.empty(M * tiles, dtype=torch.int32, device=x.device)
    _check(library().nvbe_layer_gemm_sample(_s(stream), _p(x), _p(w), _p(logits), M, N, K, _p(temperatures),
                                            _p(seeds), _p(out), _p(ps), _p(pi)))


def gemm_device_error():
    return library().nvbe_gemm_device_error()


def layer_sample(logits, temperatures, seeds, out, stream=None):
    import torch

    rows, vocab = logits.shape
    parts = library().nvbe_sample_partitions(vocab)
    ps = torch.empty(rows * parts, dtype=torch.float32, device=logits.device)
    pi = torch.empty(rows * parts, dtype=torch.int32, device=logits.device)
    _check(library().nvbe_layer_sample(_s(stream), _p(logits), _p(temperatures), _p(seeds), _p(out), _p(ps), _p(pi),
                                       rows, vocab))
