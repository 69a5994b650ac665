"""Host-side metadata of the paged attention path (libnvb_host.so), on CPU.

Known answers are the reference's own unit tests: src/model.rs:1170-1302
(flash_metadata, packed metadata) and src/runtime/tests.rs:213-256 (prefix
collision, LRU eviction). make_batch is checked with the slot / table
invariants the reference's KvRunner asserts (src/runtime/tests.rs:33-83).
"""
import random

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st


@pytest.fixture(scope="module")
def H(nvb):
    import importlib

    return importlib.import_module("nano_vllm_rs_b200.host")


def test_flash_metadata_preserves_cached_prefix_causal_offsets(H):
    b = H.Batch(positions=[256, 257, 258, 512, 513], sequence_ids=[0, 0, 0, 1, 1])
    cu, kv, mq = H.flash_metadata(b, 2)
    assert (cu, kv, mq) == ([0, 3, 5], [259, 514], 3)
    for s in range(2):
        assert kv[s] - (cu[s + 1] - cu[s]) == b.positions[cu[s]]


def test_flash_metadata_ragged_prefill_and_decode(H):
    ragged = H.Batch(positions=[0, 1, 1023, 509, 510, 511], sequence_ids=[0, 0, 1, 2, 2, 2])
    assert H.flash_metadata(ragged, 3) == ([0, 2, 3, 6], [2, 1024, 512], 3)
    decode = H.Batch(positions=[0, 255, 4095], sequence_ids=[0, 1, 2], is_decode=True)
    assert H.flash_metadata(decode, 3) == ([0, 1, 2, 3], [1, 256, 4096], 1)


@pytest.mark.parametrize("positions,seqs,n,msg", [
    ([0, 0, 1], [0, 1, 0], 2, "out of order"),
    ([0, 0], [1, 0], 2, "nonempty"),
    ([0, 0], [0, 2], 3, "nonempty"),
    ([255, 257], [0, 0], 1, "consecutive"),
    ([256, 256], [0, 0], 1, "consecutive"),
    ([2**31 - 1], [0], 1, "overflow"),
])
def test_flash_metadata_rejects_invalid_groups(H, positions, seqs, n, msg):
    with pytest.raises(H.HostError, match=msg):
        H.flash_metadata(H.Batch(positions=positions, sequence_ids=seqs), n)


def _groups_batch(H, lens, starts):
    positions, seqs = [], []
    for s, (n, p0) in enumerate(zip(lens, starts)):
        positions += range(p0, p0 + n)
        seqs += [s] * n
    return H.Batch(positions=positions, sequence_ids=seqs)


_groups = st.lists(st.tuples(st.integers(1, 40), st.integers(0, 100_000)), min_size=1, max_size=12)


@settings(max_examples=150, deadline=None)
@given(groups=_groups)
def test_flash_metadata_property_valid_groups(H, groups):
    # Any batch of nonempty, in-order groups of consecutive positions: cu_q is
    # the running row count, kv_len the group's last position + 1, max_q the
    # longest group (src/model.rs:234-267).
    lens, starts = [g[0] for g in groups], [g[1] for g in groups]
    cu, kv, mq = H.flash_metadata(_groups_batch(H, lens, starts), len(groups))
    assert cu == [0] + np.cumsum(lens).tolist()
    assert kv == [p0 + n for n, p0 in zip(lens, starts)]
    assert mq == max(lens)


@settings(max_examples=150, deadline=None)
@given(groups=_groups, pick=st.integers(0, 10**6), delta=st.sampled_from([-2, -1, 1, 2]))
def test_flash_metadata_property_rejects_a_gap(H, groups, pick, delta):
    # One position moved inside a group of two or more rows breaks the
    # consecutive run: rejected like the reference does.
    lens, starts = [g[0] for g in groups], [g[1] for g in groups]
    multi = [s for s, n in enumerate(lens) if n >= 2]
    if not multi:
        return
    b = _groups_batch(H, lens, starts)
    s = multi[pick % len(multi)]
    row = sum(lens[:s]) + 1 + (pick // 7) % (lens[s] - 1)
    b.positions[row] += delta
    with pytest.raises(H.HostError, match="consecutive"):
        H.flash_metadata(b, len(groups))


@settings(max_examples=100, deadline=None)
@given(groups=_groups.filter(lambda g: len(g) >= 2), pick=st.integers(0, 10**6))
def test_flash_metadata_property_rejects_groups_out_of_order(H, groups, pick):
    # Two groups swapped (sequence ids no longer ascending) are rejected.
    lens, starts = [g[0] for g in groups], [g[1] for g in groups]
    b = _groups_batch(H, lens, starts)
    a = pick % (len(groups) - 1)
    order = list(range(len(groups)))
    order[a], order[a + 1] = order[a + 1], order[a]
    rows = []
    for s in order:
        r0 = sum(lens[:s])
        rows += range(r0, r0 + lens[s])
    b2 = H.Batch(positions=[b.positions[r] for r in rows], sequence_ids=[b.sequence_ids[r] for r in rows])
    with pytest.raises(H.HostError):
        H.flash_metadata(b2, len(groups))


def test_packed_metadata_alignment_values_and_table_padding(H):
    layout = H.MetadataLayout(3, 2, 3)
    order = ["tokens", "positions", "sequences", "slots", "tables", "last_indices", "temperatures", "seeds"]
    for f in order:
        s, e = layout.ranges[f]
        assert s % 8 == 0 and e <= layout.bytes
    for a, b in zip(order, order[1:]):
        assert layout.ranges[a][1] <= layout.ranges[b][0]
    batch = H.Batch(token_ids=[5, 8, 13], positions=[0, 1, 0], sequence_ids=[0, 0, 1], slot_mapping=[20, 21, 40],
                    block_tables=[2, 4], table_stride=1, last_token_indices=[1, 2], temperatures=[0.0, 0.6],
                    seeds=[0x0102030405060708, 2**64 - 1])
    staging = np.full(layout.bytes, 0x55, np.uint8)
    layout.pack(staging, batch, 2, 3)

    def i32(f):
        s, e = layout.ranges[f]
        return staging[s:e].view(np.int32).tolist()

    assert i32("tokens") == [5, 8, 13]
    assert i32("positions") == [0, 1, 0]
    assert i32("tables") == [2, -1, -1, 4, -1, -1]
    s = layout.ranges["seeds"][0]
    assert staging[s:s + 8].tobytes() == (0x0102030405060708).to_bytes(8, "little")
    t = layout.ranges["temperatures"][0]
    assert staging[t + 4:t + 8].tobytes() == np.float32(0.6).tobytes()
    smaller = H.Batch(token_ids=[21], positions=[0], sequence_ids=[0], slot_mapping=[70], block_tables=[7],
                      table_stride=1)
    layout.pack(staging, smaller, 1, 3)
    tb = layout.ranges["tables"][0]
    assert staging[tb + 4:tb + 12].tolist() == [0xff] * 8


def test_packed_metadata_writes_flash_fields(H):
    layout = H.MetadataLayout(4, 2, 2)
    batch = H.Batch(token_ids=[1, 2, 3, 4], positions=[5, 6, 0, 1], sequence_ids=[0, 0, 1, 1],
                    slot_mapping=[5, 6, 256, 257], block_tables=[0, -1, 1, -1], table_stride=2)
    cu, kv, _ = H.flash_metadata(batch, 2)
    staging = np.zeros(layout.bytes, np.uint8)
    layout.pack(staging, batch, 2, 2, cu_q=cu, kv_lens=kv)
    s, e = layout.ranges["cu_q"]
    assert staging[s:e].view(np.int32).tolist() == [0, 2, 4]
    s, e = layout.ranges["kv_lens"]
    assert staging[s:e].view(np.int32).tolist() == [7, 2]


@settings(max_examples=120, deadline=None)
@given(data=st.data())
def test_packed_metadata_property_round_trip(H, data):
    # Any batch that fits the layout reads back field by field from the
    # staging bytes: the rows' tokens / positions / sequence ids / slots, each
    # sequence's table row padded with -1 (0xFF bytes) to the layout stride,
    # the samples' last indices / temperatures / seeds, cu_q and kv_lens.
    # The staging buffer starts as random bytes (a reused upload buffer).
    i32 = st.integers(-(2**31), 2**31 - 1)
    T, S, C = data.draw(st.integers(1, 48)), data.draw(st.integers(1, 8)), data.draw(st.integers(1, 12))
    layout = H.MetadataLayout(T, S, C)
    rows, n = data.draw(st.integers(1, T)), data.draw(st.integers(1, S))
    bstride, k = data.draw(st.integers(1, C)), data.draw(st.integers(0, S))
    ints = lambda m: data.draw(st.lists(i32, min_size=m, max_size=m))
    batch = H.Batch(token_ids=ints(rows), positions=ints(rows), sequence_ids=ints(rows), slot_mapping=ints(rows),
                    block_tables=data.draw(st.lists(st.integers(-1, 10**6), min_size=n * bstride,
                                                    max_size=n * bstride)),
                    table_stride=bstride, last_token_indices=ints(k),
                    temperatures=data.draw(st.lists(st.floats(0, 2, width=32), min_size=k, max_size=k)),
                    seeds=data.draw(st.lists(st.integers(0, 2**64 - 1), min_size=k, max_size=k)))
    cu, kv = ints(n + 1), ints(n)
    rng = np.random.default_rng(data.draw(st.integers(0, 2**32 - 1)))
    staging = rng.integers(0, 256, layout.bytes, dtype=np.uint8)
    layout.pack(staging, batch, n, C, cu_q=cu, kv_lens=kv)

    def field(f, count, dtype):
        s0 = layout.ranges[f][0]
        return staging[s0:s0 + count * np.dtype(dtype).itemsize].view(dtype).tolist()

    for f, want in (("tokens", batch.token_ids), ("positions", batch.positions), ("sequences", batch.sequence_ids),
                    ("slots", batch.slot_mapping), ("last_indices", batch.last_token_indices), ("cu_q", cu),
                    ("kv_lens", kv)):
        assert field(f, len(want), np.int32) == want, f
    tables = np.full((n, C), -1, np.int64)
    tables[:, :bstride] = np.asarray(batch.block_tables, np.int64).reshape(n, bstride)
    assert field("tables", n * C, np.int32) == tables.ravel().tolist()
    assert field("temperatures", k, np.float32) == np.asarray(batch.temperatures, np.float32).tolist()
    assert field("seeds", k, np.uint64) == batch.seeds


LIM = dict(max_batch_tokens=16, max_sequences=4, max_model_len=32, block_size=4, num_blocks=8, table_stride=8,
           vocab_size=100)


def _good():
    # seq 0 at positions 4..6 (pages 3, 5), seq 1 decode at position 2 (page 1)
    return H_batch(token_ids=[1, 2, 3, 4], positions=[4, 5, 6, 2], sequence_ids=[0, 0, 0, 1],
                   slot_mapping=[5 * 4 + 0, 5 * 4 + 1, 5 * 4 + 2, 1 * 4 + 2], block_tables=[3, 5, 1, -1],
                   table_stride=2, last_token_indices=[2, 3], temperatures=[0.0, 0.6], seeds=[1, 2])


H_batch = None


@pytest.fixture(autouse=True)
def _bind(H):
    global H_batch
    H_batch = H.Batch


def test_validate_batch_accepts_consistent_batch(H):
    assert H.validate_batch(_good(), **LIM) == (4, 2, 2)


@pytest.mark.parametrize("mutate,msg", [
    (lambda b: b.slot_mapping.__setitem__(1, 99), "disagrees"),
    (lambda b: b.slot_mapping.__setitem__(1, 20), "disagrees"),
    (lambda b: b.positions.__setitem__(0, 40), "max_model_len"),
    (lambda b: b.sequence_ids.__setitem__(3, 2), "outside block tables"),
    (lambda b: b.block_tables.__setitem__(1, 9), "invalid physical KV block"),
    (lambda b: b.token_ids.__setitem__(0, 100), "vocabulary"),
    (lambda b: b.last_token_indices.__setitem__(0, 4), "sample row"),
    (lambda b: b.temperatures.__setitem__(1, float("nan")), "temperature"),
    (lambda b: b.block_tables.__setitem__(0, -1), "causal context"),
])
def test_validate_batch_rejects(H, mutate, msg):
    b = _good()
    mutate(b)
    with pytest.raises(H.HostError, match=msg):
        H.validate_batch(b, **LIM)


def test_validate_batch_rejects_duplicate_slots(H):
    b = H.Batch(token_ids=[1, 2], positions=[0, 0], sequence_ids=[0, 1], slot_mapping=[4, 4], block_tables=[1, 1],
                table_stride=1)
    with pytest.raises(H.HostError, match="same KV slot"):
        H.validate_batch(b, **LIM)


def test_pool_prefix_lookup_checks_collision_tokens(H):
    # src/runtime/tests.rs:224-233
    pool = H.BlockPool(1)
    block = pool.allocate()
    pool.publish(block, [1, 2])
    pool.release(block)
    pool.force_hash_entry([3, 4], block)  # simulated hash collision
    assert pool.find_and_retain([3, 4]) is None
    assert pool.find_and_retain([1, 2]) == block


def test_pool_lru_eviction_clears_stale_keys_and_keeps_referenced_blocks(H):
    # src/runtime/tests.rs:236-256
    pool = H.BlockPool(2)
    first = pool.allocate()
    pool.publish(first, [1, 2])
    pool.release(first)
    second = pool.allocate()
    pool.publish(second, [3, 4])
    pool.release(second)
    assert pool.find_and_retain([1, 2]) == first
    assert pool.find_and_retain([1, 2]) == first
    assert pool.allocate() == second
    assert pool.find_and_retain([3, 4]) is None
    assert pool.references(first) == 2
    pool.release(first)
    assert pool.allocate() is None
    pool.release(first)
    assert pool.allocate() == first
    assert pool.cached_keys() == 0


def test_pool_prefers_empty_pages_then_least_recently_used(H):
    pool = H.BlockPool(4)
    a, b, c = pool.allocate(), pool.allocate(), pool.allocate()
    assert (a, b, c) == (0, 1, 2)
    pool.publish(a, [9])
    for x in (c, a, b):
        pool.release(x)
    assert pool.allocate() == 3          # never-used empty page first
    assert pool.allocate() == c          # then empty pages by last use
    assert pool.allocate() == b
    assert pool.allocate() == a          # the keyed page last; its key is dropped
    assert pool.find([9]) is None and pool.available() == 0 and pool.in_use() == 4
    pool.clear_cache()


def _mix(v):
    m = (1 << 64) - 1
    v = (v + 0x9E3779B97F4A7C15) & m
    v = ((v ^ (v >> 30)) * 0xBF58476D1CE4E5B9) & m
    v = ((v ^ (v >> 27)) * 0x94D049BB133111EB) & m
    return v ^ (v >> 31)


def test_sampling_seed_matches_independent_restatement(H):
    for base, rid, gen in ((42, 0, 0), (42, 7, 511), (2**64 - 1, 2**63, 3)):
        assert H.sampling_seed(base, rid, gen) == _mix(_mix(base) ^ _mix(rid) ^ _mix(gen))


@pytest.mark.parametrize("seed", range(24))
def test_make_batch_slot_and_table_invariants(H, seed):
    rng = random.Random(seed)
    bs = rng.choice([2, 4, 256])
    pool = H.BlockPool(256)
    segs = []
    for rid in range(rng.randint(1, 6)):
        n = rng.randint(1, 3 * bs + 1)
        start = rng.randint(0, n - 1)
        blocks = [pool.allocate() for _ in range((n + bs - 1) // bs)]
        segs.append(H.Segment(tokens=[rng.randint(0, 999) for _ in range(n)], blocks=blocks, start=start, end=n,
                              sample=rng.random() < 0.7, request_id=rid, generated=rng.randint(0, 9),
                              temperature=0.6))
    b = H.make_batch(segs, bs, seed=42)
    stride = max(len(s.blocks) for s in segs)
    assert b.table_stride == stride and len(b.block_tables) == stride * len(segs)
    written = set()
    for i in range(len(b.positions)):
        row, pos = b.sequence_ids[i], b.positions[i]
        page = b.block_tables[row * stride + pos // bs]
        assert page >= 0 and b.slot_mapping[i] == page * bs + pos % bs
        assert b.slot_mapping[i] not in written
        written.add(b.slot_mapping[i])
        assert b.token_ids[i] == segs[row].tokens[pos]
    for r, s in enumerate(segs):
        row = b.block_tables[r * stride:(r + 1) * stride]
        assert row[:len(s.blocks)] == s.blocks and all(x == -1 for x in row[len(s.blocks):])
    sampled = [r for r, s in enumerate(segs) if s.sample]
    assert [b.sequence_ids[i] for i in b.last_token_indices] == sampled
    assert b.seeds == [H.sampling_seed(42, segs[r].request_id, segs[r].generated) for r in sampled]
    # the batch passes the model's host validation and yields the causal metadata
    lim = dict(max_batch_tokens=len(b.positions), max_sequences=len(segs), max_model_len=4 * bs + 2, block_size=bs,
               num_blocks=256, table_stride=stride, vocab_size=1000)
    assert H.validate_batch(b, **lim)[:2] == (len(b.positions), len(segs))
    cu, kv, _ = H.flash_metadata(b, len(segs))
    assert kv == [s.end for s in segs]
    # one row's slot moved to the same offset of the next page: the row no
    # longer agrees with its table, and validation says so
    i = rng.randrange(len(b.positions))
    b.slot_mapping[i] += bs
    with pytest.raises(H.HostError, match="disagrees"):
        H.validate_batch(b, **lim)
