"""Multi-rank host logic on CPU (gloo, world size 2): kv-head shard plans,
the output all-gather order, sequence shards, and a rank that leaves before
the collective (its peer must fail with an error, not hang)."""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _load():
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    import __graft_entry__

    __graft_entry__.load_package()
    import importlib

    return importlib.import_module("nano_vllm_rs_b200.sharding")


def _gather_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        S = _load()
        shard = S.HeadShard(rank, world, kv_heads=8, q_heads=64)
        b, d = 4, 128
        # each element encodes (sequence, global query head, dim)
        heads = torch.tensor(list(shard.q_range), dtype=torch.float32)
        local = (torch.arange(b).view(b, 1, 1) * 1e4 + heads.view(1, -1, 1) * 10 +
                 torch.arange(d).view(1, 1, d) * 1e-3).float()
        full = S.gather_heads(local, shard)
        expect = (torch.arange(b).view(b, 1, 1) * 1e4 + torch.arange(64).view(1, -1, 1).float() * 10 +
                  torch.arange(d).view(1, 1, d) * 1e-3)
        ok = tuple(full.shape) == (b, 64, d) and torch.equal(full, expect)
        seqs = [list(S.sequence_shard(10, r, world)) for r in range(world)]
        q.put((rank, ok, list(shard.kv_range), list(shard.q_range), seqs))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, False, repr(e), None, None))


def test_kv_head_shards_and_gather_order_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert [r[1] for r in results] == [True, True], results
    assert results[0][2] == [0, 1, 2, 3] and results[1][2] == [4, 5, 6, 7]
    assert results[0][3] == list(range(32)) and results[1][3] == list(range(32, 64))
    assert results[0][4] == [list(range(0, 5)), list(range(5, 10))]


def _dropout_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        # leaves between steps without joining the collective
        q.put((rank, "left"))
        q.close()
        q.join_thread()
        os._exit(0)
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put((rank, "no error"))
    except Exception as e:  # the timeout surfaces as an exception
        q.put((rank, "error: " + type(e).__name__))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_that_leaves_surfaces_as_error_on_peer():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results[1] == "left"
    assert results[0].startswith("error"), results


def test_shard_plan_rejects_uneven_heads():
    S = _load()
    with pytest.raises(ValueError):
        S.HeadShard(0, 3, kv_heads=8, q_heads=64)
    assert [len(S.sequence_shard(256, r, 8)) for r in range(8)] == [32] * 8
    assert sum(len(S.sequence_shard(7, r, 3)) for r in range(3)) == 7


def test_sequence_shards_partition_every_small_batch():
    # Every batch of 0-64 sequences over 1-8 ranks: the ranks' ranges, in rank
    # order, tile [0, batch) exactly, and their sizes differ by at most one.
    S = _load()
    for world in range(1, 9):
        for batch in range(65):
            parts = [S.sequence_shard(batch, r, world) for r in range(world)]
            assert [i for p in parts for i in p] == list(range(batch)), (batch, world)
            sizes = [len(p) for p in parts]
            assert max(sizes) - min(sizes) <= 1, (batch, world)
    # kv-head shards tile the heads the same way, each rank with its GQA groups
    for world, kvh, qh in ((1, 8, 64), (2, 8, 64), (4, 8, 32), (8, 8, 64), (2, 2, 16)):
        shards = [S.HeadShard(r, world, kv_heads=kvh, q_heads=qh) for r in range(world)]
        assert [h for s in shards for h in s.kv_range] == list(range(kvh))
        assert [h for s in shards for h in s.q_range] == list(range(qh))
        for s in shards:
            assert all(q // (qh // kvh) in s.kv_range for q in s.q_range)


class _FakePeerLib:
    """Stands in for the CUDA IPC calls: a handle is the owner's pointer."""

    def peer_buffer_open(self, handle):
        return int.from_bytes(handle[:8], "little") + 1  # a mapping differs from the owner's address


def _peer_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        S = _load()
        shard = S.HeadShard(rank, world, kv_heads=8, q_heads=64)
        own = 0x1000 * (rank + 1)
        bases = S.exchange_peer_buffers(_FakePeerLib(), shard, own, own.to_bytes(64, "little"))
        q.put((rank, bases))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


def test_peer_buffer_exchange_world2():
    # each rank keeps its own pointer and maps the other's handle, in rank order
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results[0] == [0x1000, 0x2000 + 1], results
    assert results[1] == [0x1000 + 1, 0x2000], results
