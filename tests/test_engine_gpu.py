"""The Qwen3 engine on the GPU against the reference engine's own kernels.

* Layer kernels (libnvb_model.so) are bit-identical to the reference's
  (kernels/kernels.cu, built from source into oracle/_ref/libref_native.so):
  embedding, RMSNorm, add+RMSNorm, SiLU*up, row gather and the Gumbel-max
  sampler.
* BASELINE config 4's architecture (Qwen3-0.6B, 28 layers, random weights
  N(0, 0.02)), 6 prompts x 64 sampled tokens (temperature 0.6 Gumbel-max,
  seed 42, ignore_eos) through chunked prefill, multi-page contexts and
  graph-replayed decode: run in lockstep with the reference's forward
  (tests/ref_model.py) on its native attention backend, this engine's
  tokens equal the reference's except at near ties that the step's logit
  difference provably explains, and it agrees with the native backend at
  least about as well as the reference's own FA2 backend does. Exact token
  equality over 64 free-running steps is not a property two different
  attention algorithms can have at BF16 on near-uniform random-weight
  logits (the reference records the same for its FA2 backend,
  ATTENTION.md:5, 52); the free-running test checks the agreement prefix.
* Graph-replayed decode gives the same tokens as eager decode.
"""
import pytest
import torch

import __graft_entry__
from conftest import as_f32, bits

pytestmark = pytest.mark.gpu

pkg = __graft_entry__.load_package()
M = pkg.model
E = pkg.engine


def _stream_ref(ref_native):
    import ctypes

    sp = ctypes.c_void_p()
    ref_native.L.nv_stream(ref_native.ctx, ctypes.byref(sp))
    return torch.cuda.ExternalStream(sp.value)


@pytest.fixture(scope="module")
def ref_layers(ref_native):
    from ref_model import declare

    declare(ref_native.L)
    return ref_native


def _ref(ref_native, name, *args):
    torch.cuda.synchronize()
    ref_native.call(name, *args)


def test_layer_embedding_and_gather_bit_identical(ref_layers):
    g = torch.Generator(device="cuda").manual_seed(1)
    vocab, hidden, rows = 5000, 1024, 77
    weight = torch.randn(vocab, hidden, generator=g, device="cuda").bfloat16()
    tokens = torch.randint(0, vocab, (rows,), generator=g, device="cuda", dtype=torch.int32)
    tokens[3], tokens[10] = -1, vocab  # out of range: zero rows
    mine, ref = torch.empty(rows, hidden, dtype=torch.bfloat16, device="cuda"), torch.empty(rows, hidden,
                                                                                             dtype=torch.bfloat16,
                                                                                             device="cuda")
    M.layer_embedding(tokens, weight, mine)
    _ref(ref_layers, "nv_embedding", tokens, weight, ref, rows, hidden, vocab)
    assert (bits(mine) == bits(ref)).all()
    idx = torch.tensor([5, 0, 76, -1, 80, 33], dtype=torch.int32, device="cuda")
    gm, gr = (torch.empty(6, hidden, dtype=torch.bfloat16, device="cuda") for _ in range(2))
    M.layer_gather(mine, idx, gm)
    _ref(ref_layers, "nv_gather", mine, idx, gr, 6, hidden, rows)
    assert (bits(gm) == bits(gr)).all()


@pytest.mark.parametrize("hidden,rows,scale", [(1024, 300, 1.0), (1024, 5, 30.0), (4096, 64, 0.02), (1000, 9, 1.0)])
def test_layer_rms_and_add_rms_bit_identical(ref_layers, hidden, rows, scale):
    g = torch.Generator(device="cuda").manual_seed(hidden + rows)
    x = (torch.randn(rows, hidden, generator=g, device="cuda") * scale).bfloat16()
    res = (torch.randn(rows, hidden, generator=g, device="cuda") * scale).bfloat16()
    w = (1 + 0.02 * torch.randn(hidden, generator=g, device="cuda")).bfloat16()
    mine, ref = torch.empty_like(x), torch.empty_like(x)
    M.layer_rms(x, w, mine, 1e-6)
    _ref(ref_layers, "nv_rms", x, w, ref, rows, hidden, 1e-6)
    assert (bits(mine) == bits(ref)).all()
    r_mine, r_ref = res.clone(), res.clone()
    M.layer_add_rms(x, r_mine, w, mine, 1e-6)
    _ref(ref_layers, "nv_add_rms", x, r_ref, w, ref, rows, hidden, 1e-6)
    assert (bits(r_mine) == bits(r_ref)).all()
    assert (bits(mine) == bits(ref)).all()


def test_layer_silu_mul_bit_identical(ref_layers):
    g = torch.Generator(device="cuda").manual_seed(3)
    rows, inter = 129, 3072
    packed = (torch.randn(rows, 2 * inter, generator=g, device="cuda") * 4).bfloat16()
    packed[0, :8] = torch.tensor([0.0, -0.0, 88.0, -88.0, 100.0, -100.0, 1e-30, -1e-30]).bfloat16()
    mine, ref = (torch.empty(rows, inter, dtype=torch.bfloat16, device="cuda") for _ in range(2))
    M.layer_silu_mul(packed, mine)
    _ref(ref_layers, "nv_silu", packed, ref, rows, inter)
    assert (bits(mine) == bits(ref)).all()


@pytest.mark.parametrize("vocab", [151936, 5000, 2047])
def test_layer_sample_matches_reference_sampler(ref_layers, vocab):
    g = torch.Generator(device="cuda").manual_seed(vocab)
    rows = 40
    logits = (torch.randn(rows, vocab, generator=g, device="cuda") * 2).bfloat16()
    logits[1, :] = 0.5                      # all tied: lowest id under greedy
    logits[2, 7] = logits[2, vocab - 3] = 40.0  # a tie at the top
    temps = torch.tensor([0.0, 0.0, 0.0] + [0.6, 1.0, 0.0, 2.5] * 9 + [0.6], dtype=torch.float32, device="cuda")
    seeds = torch.randint(-2**62, 2**62, (rows,), generator=g, device="cuda", dtype=torch.int64)
    mine = torch.empty(rows, dtype=torch.int32, device="cuda")
    M.layer_sample(logits, temps, seeds, mine)
    parts = -(-vocab // 2048)
    ps = torch.empty(rows * parts, dtype=torch.float32, device="cuda")
    pi = torch.empty(rows * parts, dtype=torch.int32, device="cuda")
    ref_par, ref_one = (torch.empty(rows, dtype=torch.int32, device="cuda") for _ in range(2))
    _ref(ref_layers, "nv_sample_parallel", logits, temps, seeds, ref_par, ps, pi, rows, vocab)
    _ref(ref_layers, "nv_sample", logits, temps, seeds, ref_one, rows, vocab)
    assert mine.tolist() == ref_par.tolist() == ref_one.tolist()
    assert mine[1].item() == 0 and mine[2].item() == 7


# ------------------------------------------------------------------ engine
CONFIG = M.Qwen3Config()  # Qwen3-0.6B shape


@pytest.fixture(scope="module")
def weights():
    return M.random_weights(CONFIG, seed=0)


def _requests(n_tokens, max_tokens=64, seed=11):
    g = torch.Generator().manual_seed(seed)
    return [E.Request(id=100 + i, prompt_token_ids=torch.randint(0, CONFIG.vocab_size, (n,), generator=g).tolist(),
                      max_tokens=max_tokens, temperature=0.6, ignore_eos=True) for i, n in enumerate(n_tokens)]


SCHED = dict(block_size=256, num_blocks=48, max_sequences=6, max_model_len=1024, max_batch_tokens=512)
PROMPTS = [300, 37, 600, 129, 256, 700]  # chunked prefill (budget 512), page boundaries, mixed lengths


def _options(graphs=True):
    s = SCHED
    return M.ModelOptions(device=0, block_size=s["block_size"], num_blocks=s["num_blocks"],
                          max_batch_tokens=s["max_batch_tokens"], max_sequences=s["max_sequences"],
                          max_model_len=s["max_model_len"], cuda_graphs=graphs)


def _ours(weights, reqs, graphs=True):
    model = M.Qwen3Model(CONFIG, _options(graphs), weights)
    engine = E.LlmEngine(E.SchedulerConfig(**SCHED), model)
    out = engine.generate(reqs, 42)
    graphs_made = model.graph_count()
    engine.close()
    model.close()
    return out, graphs_made


def test_engine_tokens_track_reference_native_backend_for_64_steps(weights, ref_native, ref_flash):
    """Lockstep over 6 prompts x 64 sampled tokens (tests/lockstep.py): the
    reference native backend leads; this library's engine and, as the
    calibration, the reference's own FA2 backend follow on the same
    contexts. Every token that differs from the native backend's must be a
    near tie explained by that step's logit difference; the logits must stay
    close; and this engine must agree with the native backend at least about
    as well as the reference's FA2 backend does (both round P to BF16 for
    the PV product, the native kernel does not)."""
    import json
    import os

    from lockstep import Lockstep, OursRunner
    from ref_model import RefRunner

    reqs = _requests(PROMPTS)
    model = M.Qwen3Model(CONFIG, _options(True), weights)
    native = RefRunner(ref_native, CONFIG, _options(False), weights)
    flash = RefRunner(ref_native, CONFIG, _options(False), weights, flash=ref_flash)
    hybrid = RefRunner(ref_native, CONFIG, _options(False), weights, nvb=pkg)
    lock = Lockstep(native, {"ours": OursRunner(pkg, model), "reference_fa2": flash,
                             "reference_with_our_attention": hybrid})
    out = E.LlmEngine(E.SchedulerConfig(**SCHED), lock).generate(reqs, 42)
    graphs = model.graph_count()
    model.close()
    s = lock.summary()
    report = os.environ.get("NVB_PARITY_JSON")
    if report:
        with open(report, "w") as f:
            json.dump(s, f, indent=1, default=float)
    print(json.dumps({k: v if not isinstance(v, dict) else {a: b for a, b in v.items() if a != "unexplained"}
                      for k, v in s.items()}, default=float))
    assert graphs >= 1
    assert s["samples"] == 6 * 64 and all(len(o.token_ids) == 64 for o in out.outputs)
    ours, fa2 = s["ours"], s["reference_fa2"]
    assert not ours["unexplained"], ours["unexplained"]
    assert not fa2["unexplained"], fa2["unexplained"]
    # Calibrated on the reference's FA2 backend against its native backend on
    # the same contexts (mean 0.0069, max 0.055 logit; 2 of 384 tokens):
    # this engine must be at most a quarter worse on average.
    assert ours["max_logit_delta"] <= 0.125
    assert ours["mean_logit_err"] <= 1.25 * fa2["mean_logit_err"] + 1e-4
    assert ours["match_rate"] >= 0.98


def test_engine_free_running_tokens_follow_reference_until_a_near_tie(weights, ref_native):
    """Free-running generation (each engine feeds back its own tokens): the
    tokens agree with the reference native backend's from the start; the
    first difference, if any, must come no earlier than the first step at
    which the lockstep comparison above would also see a near tie. Here it
    is checked per request as: the common prefix is a prefix of both, and
    at least the first 8 tokens agree."""
    from ref_model import RefRunner

    reqs = _requests(PROMPTS)
    mine, _ = _ours(weights, reqs)
    ref = E.LlmEngine(E.SchedulerConfig(**SCHED), RefRunner(ref_native, CONFIG, _options(False), weights)).generate(
        reqs, 42)
    agree = []
    for a, b in zip(mine.outputs, ref.outputs):
        n = next((i for i, (x, y) in enumerate(zip(a.token_ids, b.token_ids)) if x != y), len(a.token_ids))
        agree.append(n)
    print("free-running agreement per request (tokens):", agree)
    assert min(agree) >= 8, agree


def test_graph_replay_matches_eager_decode(weights):
    reqs = _requests([200, 513, 64], max_tokens=24, seed=5)
    g_out, g_count = _ours(weights, reqs, graphs=True)
    e_out, e_count = _ours(weights, reqs, graphs=False)
    assert g_count >= 1 and e_count == 0
    assert [o.token_ids for o in g_out.outputs] == [o.token_ids for o in e_out.outputs]


def test_prefill_logits_close_to_reference(weights, ref_native):
    from ref_model import RefRunner

    reqs = _requests([400, 77, 900], max_tokens=1, seed=9)
    model = M.Qwen3Model(CONFIG, _options(), weights)
    engine = E.LlmEngine(E.SchedulerConfig(**SCHED), model)
    engine.generate(reqs, 42)
    mine = model.last_logits().float()
    ref_runner = RefRunner(ref_native, CONFIG, _options(False), weights)
    E.LlmEngine(E.SchedulerConfig(**SCHED), ref_runner).generate(reqs, 42)
    ref = ref_runner.last_logits().float()
    engine.close()
    model.close()
    assert mine.shape == ref.shape
    err = (mine - ref).abs()
    # BF16 logits of magnitude ~1: different attention rounding moves them by
    # a few ulp after 28 layers (the lockstep test above calibrates this
    # against the reference's own FA2 backend)
    assert err.max().item() <= 0.125 and err.mean().item() <= 1e-2, (err.max().item(), err.mean().item())
    assert (mine.argmax(-1) == ref.argmax(-1)).all()


def test_mixed_batches_track_reference_native_backend(weights, ref_native):
    """Mixed forwards (decode rows and prefill chunks in one forward, the
    scheduler's mixed_batches) in lockstep with the reference's native
    forward on the same batches: 10 requests through 4 sequence slots, so
    requests are admitted and prefilled while others decode. The batches
    really mix; every differing token is a near tie explained by the step's
    logit difference, and the logits stay as close as in the lockstep test
    above."""
    from lockstep import Lockstep, OursRunner
    from ref_model import RefRunner

    sched = dict(SCHED, max_sequences=4, max_batch_tokens=384, mixed_batches=True)
    reqs = _requests([300, 37, 600, 129, 256, 700, 90, 410, 15, 333], max_tokens=16, seed=23)
    model = M.Qwen3Model(CONFIG, _options(True), weights)
    native = RefRunner(ref_native, CONFIG, _options(False), weights)
    lock = Lockstep(native, {"ours": OursRunner(pkg, model)})
    out = E.LlmEngine(E.SchedulerConfig(**sched), lock).generate(reqs, 42)
    model.close()
    s = lock.summary()["ours"]
    assert out.stats["mixed_steps"] > 0
    assert all(len(o.token_ids) == 16 for o in out.outputs)
    assert not s["unexplained"], s["unexplained"]
    assert s["max_logit_delta"] <= 0.125
    assert s["match_rate"] >= 0.97
