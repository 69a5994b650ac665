"""Scheduler of the continuous-batching engine (engine.cpp) on CPU.

Each case restates one of the reference's own scheduler tests
(src/runtime/tests.rs) with the same token-level KV simulator as the runner:
every sampled token is a hash of the whole context read back through the
batch's physical page table, so a stale, shared or overwritten page changes
the output. Expected outputs come from running each request alone on the
same hash (src/runtime/tests.rs:104-116).
"""
import math

import pytest

import __graft_entry__

E = __graft_entry__.load_package().engine
M64 = (1 << 64) - 1


def reference_next(context, temperature, seed):
    """src/runtime/tests.rs:25-31."""
    value = 7
    for t in context:
        value = (value * 31 + int(t)) & M64
    rnd = int(seed) if temperature > 0 else 0
    return (value ^ rnd) % 1000 + 1


class KvRunner:
    """src/runtime/tests.rs:4-88: checks each batch's slots against its page
    table, writes the batch's tokens into a simulated cache, and samples from
    the context read back through the table."""

    def __init__(self, config, fail_at=None, eos=None):
        self.bs = config.block_size
        self.kv = [None] * (config.block_size * config.num_blocks)
        self.batches = []
        self.fail_at = fail_at
        self.eos = eos

    def run(self, batch):
        if self.fail_at == len(self.batches):
            raise RuntimeError("injected model failure")
        n = len(batch.token_ids)
        assert len(batch.positions) == n and len(batch.sequence_ids) == n and len(batch.slot_mapping) == n
        assert len(batch.last_token_indices) == len(batch.temperatures) == len(batch.seeds)
        assert batch.sequence_count() > 0
        written = set()
        for i in range(n):
            slot, row, pos = int(batch.slot_mapping[i]), int(batch.sequence_ids[i]), int(batch.positions[i])
            physical = int(batch.block_tables[row * batch.table_stride + pos // self.bs])
            assert physical >= 0
            assert slot == physical * self.bs + pos % self.bs
            assert slot not in written, "two batch rows overwrite the same KV slot"
            written.add(slot)
            self.kv[slot] = int(batch.token_ids[i])
        samples = []
        for k, index in enumerate(batch.last_token_indices):
            row, end = int(batch.sequence_ids[index]), int(batch.positions[index])
            context = []
            for pos in range(end + 1):
                physical = int(batch.block_tables[row * batch.table_stride + pos // self.bs])
                assert physical >= 0
                v = self.kv[physical * self.bs + pos % self.bs]
                assert v is not None, "attention read uninitialized KV"
                context.append(v)
            samples.append(self.eos if self.eos is not None else
                           reference_next(context, float(batch.temperatures[k]), int(batch.seeds[k])))
        self.batches.append(batch)
        return samples


def config(**kw):
    base = dict(block_size=2, num_blocks=32, max_sequences=4, max_model_len=32, max_batch_tokens=16,
                prefix_caching=True, eos_token_id=None)
    base.update(kw)
    return E.SchedulerConfig(**base)


def request(id_, tokens, max_tokens, **kw):
    return E.Request(id=id_, prompt_token_ids=list(tokens), max_tokens=max_tokens, **kw)


def expected(req, seed):
    context = list(req.prompt_token_ids)
    for step in range(req.max_tokens):
        context.append(reference_next(context, req.temperature, E.sampling_seed(seed, req.id, step)))
    return context[len(req.prompt_token_ids):]


def engine_for(cfg, **runner_kw):
    runner = KvRunner(cfg, **runner_kw)
    return E.LlmEngine(cfg, runner), runner


def test_mixed_lengths_match_sequential_reference_and_release_all_blocks():
    cfg = config()
    engine, runner = engine_for(cfg)
    reqs = [request(11, [1, 2, 3], 4), request(12, [5], 2), request(13, [8, 9, 10, 11, 12], 3),
            request(14, [15, 16], 1), request(15, [19, 20, 21, 22], 2)]
    result = engine.generate(reqs, 123)
    for out, req in zip(result.outputs, reqs):
        assert out.id == req.id
        assert out.token_ids == expected(req, 123)
        assert len(out.inter_token_latencies_ms) == req.max_tokens - 1
        assert out.latency_ms >= out.ttft_ms
    assert result.stats["input_tokens"] == 15
    assert result.stats["output_tokens"] == 12
    assert result.stats["decode_steps"] > 0
    assert any(b.sequence_count() > 1 for b in runner.batches)
    assert engine.blocks_in_use() == 0


def test_chunked_prefill_obeys_token_budget_and_does_not_sample_early():
    cfg = config(max_batch_tokens=2)
    engine, runner = engine_for(cfg)
    req = request(1, [1, 2, 3, 4, 5, 6, 7], 3)
    result = engine.generate([req], 1)
    assert result.outputs[0].token_ids == expected(req, 1)
    assert result.stats["prefill_tokens"] == 7
    assert result.stats["prefill_steps"] == 4
    assert all(len(b.token_ids) <= 2 for b in runner.batches)
    assert all(len(b.last_token_indices) == 0 for b in runner.batches[:3])


def test_warm_prefix_is_shared_and_final_prompt_token_is_recomputed():
    cfg = config()
    engine, runner = engine_for(cfg)
    req = request(1, [1, 2, 3, 4, 5, 6], 1)
    cold = engine.generate([req], 1)
    warm = engine.generate([req, request(2, [1, 2, 3, 4, 5, 6], 1)], 1)
    assert warm.stats["cached_tokens"] == 8
    assert warm.stats["prefill_tokens"] == 4
    assert cold.outputs[0].token_ids == warm.outputs[0].token_ids == warm.outputs[1].token_ids
    batch = runner.batches[-1]
    s = batch.table_stride
    assert batch.sequence_count() == 2
    assert batch.block_tables[0] == batch.block_tables[s]
    assert batch.block_tables[1] == batch.block_tables[s + 1]
    assert batch.block_tables[2] != batch.block_tables[s + 2]
    assert engine.blocks_in_use() == 0
    engine.clear_prefix_cache()
    assert engine.cached_keys() == 0
    cleared = engine.generate([req], 1)
    assert cleared.stats["cached_tokens"] == 0


def test_prefix_lookup_checks_entire_context():
    cfg = config()
    engine, _ = engine_for(cfg)
    engine.generate([request(1, [1, 2, 7, 8, 9], 1)], 1)
    different = request(2, [3, 4, 7, 8, 9], 1)
    out = engine.generate([different], 1)
    assert out.stats["cached_tokens"] == 0
    assert out.outputs[0].token_ids == expected(different, 1)


def test_capacity_pressure_preempts_and_recomputes_without_losing_output():
    cfg = config(num_blocks=4, max_sequences=3, max_batch_tokens=4, max_model_len=8, prefix_caching=False)
    engine, _ = engine_for(cfg)
    reqs = [request(1, [1, 2], 6), request(2, [3, 4], 6), request(3, [5, 6], 6)]
    out = engine.generate(reqs, 4)
    assert out.stats["preemptions"] > 0
    assert out.stats["output_tokens"] == 18
    assert out.stats["peak_kv_blocks"] <= cfg.num_blocks
    for req, o in zip(reqs, out.outputs):
        assert o.token_ids == expected(req, 4)
    assert engine.blocks_in_use() == 0


def test_a_waiting_prefill_does_not_evict_established_decode_work():
    cfg = config(block_size=2, num_blocks=4, max_sequences=2, max_batch_tokens=16, max_model_len=16,
                 prefix_caching=False)
    reqs = [request(1, [1, 2, 3, 4], 4), request(2, [5], 1), request(3, [6, 7, 8, 9, 10, 11], 1)]
    engine, runner = engine_for(cfg)
    out = engine.generate(reqs, 5)
    assert out.stats["preemptions"] == 0
    assert out.stats["prefill_tokens"] == 11
    assert out.stats["output_tokens"] == 6
    assert out.outputs[0].latency_ms <= out.outputs[2].ttft_ms
    assert all(b.sequence_count() <= cfg.max_sequences for b in runner.batches)
    for req, o in zip(reqs, out.outputs):
        assert o.token_ids == expected(req, 5)
    assert engine.blocks_in_use() == 0


def test_admission_accounts_for_live_shared_prefixes_at_capacity():
    cfg = config(block_size=2, num_blocks=4, max_sequences=2, max_batch_tokens=4, max_model_len=8)
    engine, runner = engine_for(cfg)
    reqs = [request(1, [1, 2, 3, 4, 5], 3), request(2, [1, 2, 3, 4, 6], 1)]
    out = engine.generate(reqs, 0)
    assert out.stats["cached_tokens"] == 4
    assert out.stats["prefill_tokens"] == 6
    assert out.stats["preemptions"] == 0
    assert any(b.sequence_count() == 2 for b in runner.batches)
    for req, o in zip(reqs, out.outputs):
        assert o.token_ids == expected(req, 0)
    assert engine.blocks_in_use() == 0


@pytest.mark.parametrize("max_sequences", [1, 2, 5])
@pytest.mark.parametrize("max_batch_tokens", [1, 3, 10])
@pytest.mark.parametrize("prefix_caching", [False, True])
def test_seed_is_independent_of_chunking_queueing_cache_and_preemption(max_sequences, max_batch_tokens,
                                                                        prefix_caching):
    reqs = [request(i, [1, 2, 3], 5, temperature=0.7) for i in range(1, 6)]
    cfg = config(num_blocks=4, max_model_len=8, max_sequences=max_sequences, max_batch_tokens=max_batch_tokens,
                 prefix_caching=prefix_caching)
    engine, _ = engine_for(cfg)
    for _ in range(2):
        out = engine.generate(reqs, 99)
        for req, o in zip(reqs, out.outputs):
            assert o.token_ids == expected(req, 99)


@pytest.mark.parametrize("mixed", [False, True])
def test_mixed_batches_keep_outputs_and_budget(mixed):
    # Eight requests through four sequence slots: sequences are admitted
    # while others decode. Mixed forwards must give the same tokens (the
    # runner's hash reads every context back through the page tables),
    # respect the token budget, and decode in the forwards that prefill.
    cfg = config(max_sequences=4, max_batch_tokens=6, num_blocks=48, mixed_batches=mixed)
    engine, runner = engine_for(cfg)
    reqs = [request(i, list(range(i, i + 2 + i % 5)), 3 + i % 4, temperature=0.5) for i in range(1, 9)]
    out = engine.generate(reqs, 77)
    for req, o in zip(reqs, out.outputs):
        assert o.token_ids == expected(req, 77)
    assert all(len(b.token_ids) <= cfg.max_batch_tokens for b in runner.batches)
    st = out.stats
    assert st["prefill_tokens"] + st["decode_tokens"] == sum(len(b.token_ids) for b in runner.batches)
    assert st["prefill_steps"] + st["decode_steps"] + st["mixed_steps"] == len(runner.batches)
    if mixed:
        assert st["mixed_steps"] > 0 and st["mixed_seconds"] > 0
    else:
        assert st["mixed_steps"] == 0
    assert engine.blocks_in_use() == 0


def test_mixed_batches_take_fewer_forwards_and_survive_preemption():
    reqs = [request(i, [i, i + 1, i + 2], 6) for i in range(1, 7)]
    forwards = {}
    for mixed in (False, True):
        cfg = config(num_blocks=6, max_sequences=3, max_batch_tokens=4, max_model_len=10, prefix_caching=False,
                     mixed_batches=mixed)
        engine, runner = engine_for(cfg)
        out = engine.generate(reqs, 3)
        for req, o in zip(reqs, out.outputs):
            assert o.token_ids == expected(req, 3)
        assert engine.blocks_in_use() == 0
        forwards[mixed] = len(runner.batches)
    assert forwards[True] < forwards[False]


def test_eos_stops_generation_and_ignore_eos_preserves_length():
    cfg = config(eos_token_id=42)
    engine, _ = engine_for(cfg, eos=42)
    out = engine.generate([request(1, [10], 4), request(2, [20], 4, ignore_eos=True)], 0)
    assert out.outputs[0].token_ids == [42]
    assert out.outputs[0].finish_reason == "eos"
    assert out.outputs[1].token_ids == [42] * 4
    assert out.outputs[1].finish_reason == "length"
    assert engine.blocks_in_use() == 0


def test_model_failure_releases_pins_invalidates_cache_and_poisons_engine():
    cfg = config()
    engine, _ = engine_for(cfg, fail_at=1)
    with pytest.raises(E.EngineError, match="injected model failure"):
        engine.generate([request(1, [1, 2, 3], 4)], 0)
    assert engine.blocks_in_use() == 0
    assert engine.cached_keys() == 0
    with pytest.raises(E.EngineError, match="unusable"):
        engine.generate([request(2, [1], 1)], 0)


def test_invalid_requests_fail_before_running_and_empty_batch_is_valid():
    cfg = config(num_blocks=2, max_model_len=16)
    engine, runner = engine_for(cfg)
    bad = [request(1, [], 1), request(1, [1], 0), request(1, [1], 2**64 - 1), request(1, [1, 2, 3, 4], 3),
           request(1, [2**32 - 1], 1), request(1, [1], 1, temperature=math.nan)]
    for req in bad:
        with pytest.raises(E.EngineError):
            engine.generate([req], 0)
    with pytest.raises(E.EngineError, match="duplicate"):
        engine.generate([request(1, [1], 1), request(1, [2], 1)], 0)
    assert runner.batches == []
    out = engine.generate([], 0)
    assert out.outputs == []
    assert out.stats["output_tokens"] == 0
    assert math.isfinite(out.stats["output_tokens_per_second"])
    for kw in (dict(block_size=0), dict(num_blocks=0), dict(max_batch_tokens=0), dict(max_sequences=0),
               dict(num_blocks=2**64 - 1)):
        with pytest.raises(E.EngineError):
            config(**kw).validate()
