"""Multi-GPU decode over kv-head shards with the combine fused into the
all-gather (nvb_paged_decode_gather).

One GPU: world 1 (the barrier waits only on this rank's own flag), both
combine forms (split partials, and the single-split copy), two epochs in a
row, against nvb_paged_fwd on the same inputs. Two GPUs (skipped with
fewer): two processes, each holding half of the kv heads, must both end with
the whole-batch output of a single-GPU decode. Tolerance: the decode tests'
max-abs 2e-2 / mean-abs 2e-3 (the split counts differ, so rounding does).
"""
import os
import socket
from datetime import timedelta

import pytest
import torch

from conftest import as_f32, assert_close

pytestmark = pytest.mark.gpu


def _reference(nvb, case, splits):
    out = torch.empty_like(case.q)
    la, oa = nvb.splitkv_scratch(splits, case.batch, case.q_heads, "cuda") if splits > 1 else (None, None)
    nvb.paged_fwd(case.q, case.k, case.v, out, case.cu_q, case.kv_lens, case.block_table, batch=case.batch, max_q=1,
                  max_k=int(case.kv_lens.max()), q_heads=case.q_heads, kv_heads=case.kv_heads,
                  block_size=case.block_size, table_stride=case.table_stride, num_blocks=case.num_blocks,
                  num_splits=splits, lse_accum=la, out_accum=oa)
    return out


# 12 / 24 / 74 splits: the combine shared by 2 / 4 / 8 warps per item (74, the
# config-5 shard of 8 GPUs, leaves the shortest sequence's last splits empty).
@pytest.mark.parametrize("splits", [1, 6, 12, 24, 74])
def test_gather_world1_matches_paged_fwd(nvb, splits):
    import importlib

    S = importlib.import_module("nano_vllm_rs_b200.sharding")
    case = nvb.workloads.paged_case([3000, 1200, 5000], q_heads=32, kv_heads=8, seed=31)
    ref = _reference(nvb, case, splits)
    b, qh = case.batch, case.q_heads
    out_bytes = b * qh * 128 * 2
    ptr, _handle = nvb.peer_buffer_create(256 + 2 * out_bytes)
    try:
        la, oa = nvb.splitkv_scratch(splits, b, qh, "cuda") if splits > 1 else (None, None)
        local = torch.empty_like(case.q)
        for epoch in (1, 2):
            slot = ptr + 256 + (epoch & 1) * out_bytes
            nvb.paged_decode_gather(case.q, case.k, case.v, local, case.cu_q, case.kv_lens, case.block_table,
                                    batch=b, max_k=int(case.kv_lens.max()), q_heads=qh, kv_heads=case.kv_heads,
                                    block_size=case.block_size, table_stride=case.table_stride,
                                    num_blocks=case.num_blocks, num_splits=splits, lse_accum=la, out_accum=oa,
                                    peer_out=[slot], peer_flag=[ptr], rank=0, epoch=epoch)
            torch.cuda.synchronize()
            assert nvb.device_error() == 0
            got = torch.as_tensor(S._DeviceArray(slot, (b, qh, 128), "<i2"), device="cuda").view(torch.bfloat16)
            assert_close(as_f32(got), as_f32(ref), 2e-2, 2e-3, what=f"world 1, {splits} splits, epoch {epoch}")
    finally:
        nvb.peer_buffer_free(ptr)


@pytest.mark.parametrize("splits", [1, 6, 74])
def test_capturable_gather_world1_graph_replay(nvb, splits):
    """The capturable form: eager steps, then one captured step replayed
    three times; the device epoch picks the output set (odd steps set 1),
    and every step matches nvb_paged_fwd."""
    import importlib

    S = importlib.import_module("nano_vllm_rs_b200.sharding")
    case = nvb.workloads.paged_case([3000, 1200, 5000], q_heads=32, kv_heads=8, seed=32)
    ref = _reference(nvb, case, splits)
    shard = S.HeadShard(0, 1, kv_heads=8, q_heads=32)
    run = S.KvHeadShardedDecode(nvb, shard, batch=case.batch, block_size=case.block_size,
                                table_stride=case.table_stride, num_blocks=case.num_blocks,
                                max_k=int(case.kv_lens.max()), device=torch.device("cuda"), num_splits=splits)
    try:
        seen = []
        for step in range(1, 3):
            got = run(case.q, case.k, case.v, case.cu_q, case.kv_lens, case.block_table)
            torch.cuda.synchronize()
            assert got.data_ptr() == run.views[step & 1].data_ptr()
            assert_close(as_f32(got), as_f32(ref), 2e-2, 2e-3, what=f"eager step {step}")
            seen.append(got.data_ptr())
        graph = run.capture(case.q, case.k, case.v, case.cu_q, case.kv_lens, case.block_table)
        for step in range(3, 6):
            run.views[step & 1].zero_()
            got = run.replay(graph)
            torch.cuda.synchronize()
            assert got.data_ptr() == run.views[step & 1].data_ptr()
            assert_close(as_f32(got), as_f32(ref), 2e-2, 2e-3, what=f"replayed step {step}")
        assert nvb.device_error() == 0
        counter = torch.as_tensor(S._DeviceArray(run.flag_ptrs[0] + 4, (1,), "<i4"), device="cuda")
        assert int(counter.item()) == 5  # slot `world` of the flags: the device epoch
        del graph
    finally:
        run.close()


def test_gather_rejects_bad_arguments(nvb):
    case = nvb.workloads.paged_case([300], q_heads=16, kv_heads=8, seed=2)
    local = torch.empty_like(case.q)
    for kwargs, what in ((dict(peer_out=[1] * 9, peer_flag=[1] * 9, rank=0), "world 9"),
                         (dict(peer_out=[1, 1], peer_flag=[1, 1], rank=2), "rank outside world")):
        with pytest.raises(nvb.NvbError):
            nvb.paged_decode_gather(case.q, case.k, case.v, local, case.cu_q, case.kv_lens, case.block_table,
                                    batch=1, max_k=300, q_heads=16, kv_heads=8, block_size=case.block_size,
                                    table_stride=case.table_stride, num_blocks=case.num_blocks, num_splits=1,
                                    lse_accum=None, out_accum=None, epoch=1, check=False, **kwargs)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port, q):
    try:
        import sys
        from pathlib import Path

        import torch.distributed as dist

        root = Path(__file__).resolve().parents[1]
        sys.path.insert(0, str(root))
        sys.path.insert(0, str(root / "tests"))
        import __graft_entry__

        nvb = __graft_entry__.load_package()
        from nano_vllm_rs_b200 import sharding as S

        torch.cuda.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        W = nvb.workloads
        lens = [4096, 1500, 7000, 256]
        full = W.paged_case(lens, q_heads=64, kv_heads=8, seed=77, device="cuda")  # same on both ranks
        ref = _reference(nvb, full, 1).float().cpu()
        shard = S.HeadShard(rank, world, kv_heads=8, q_heads=64)
        kr, qr = shard.kv_range, shard.q_range
        q_l = full.q[:, qr.start:qr.stop].contiguous()
        k_l = full.k[:, :, kr.start:kr.stop].contiguous()
        v_l = full.v[:, :, kr.start:kr.stop].contiguous()
        run = S.KvHeadShardedDecode(nvb, shard, batch=full.batch, block_size=full.block_size,
                                    table_stride=full.table_stride, num_blocks=full.num_blocks, max_k=max(lens),
                                    device=torch.device("cuda", rank))
        errs = []
        for _ in range(3):  # three epochs: both output buffers, one reused
            got = run(q_l, k_l, v_l, full.cu_q, full.kv_lens, full.block_table)
            torch.cuda.synchronize()
            errs.append(float((got.float().cpu() - ref).abs().max()))
        graph = run.capture(q_l, k_l, v_l, full.cu_q, full.kv_lens, full.block_table)
        for _ in range(3):  # the same step replayed from a CUDA graph
            got = run.replay(graph)
            torch.cuda.synchronize()
            errs.append(float((got.float().cpu() - ref).abs().max()))
        del graph
        dev_err = nvb.device_error()
        dist.barrier()
        run.close()
        dist.destroy_process_group()
        q.put((rank, errs, dev_err, run.splits))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), -1, 0))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_gather_two_ranks_match_single_gpu_decode():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, errs, dev_err, splits in results:
        assert dev_err == 0, (rank, errs, dev_err)
        assert isinstance(errs, list) and max(errs) <= 2e-2, (rank, errs, splits)


def _two_gpu_stress_worker(rank, world, port, q, steps):
    try:
        import sys
        from pathlib import Path

        import torch.distributed as dist

        root = Path(__file__).resolve().parents[1]
        sys.path.insert(0, str(root))
        sys.path.insert(0, str(root / "tests"))
        import __graft_entry__

        nvb = __graft_entry__.load_package()
        from nano_vllm_rs_b200 import sharding as S

        torch.cuda.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        W = nvb.workloads
        lens = [9000, 3100, 6500, 700]
        shard = S.HeadShard(rank, world, kv_heads=8, q_heads=64)
        kr, qr = shard.kv_range, shard.q_range
        sets, refs = [], []
        for seed in (501, 502, 503):
            full = W.paged_case(lens, q_heads=64, kv_heads=8, seed=seed, device="cuda")
            refs.append(_reference(nvb, full, 1).float().cpu())
            sets.append((full.q[:, qr.start:qr.stop].contiguous(), full.k[:, :, kr.start:kr.stop].contiguous(),
                         full.v[:, :, kr.start:kr.stop].contiguous(), full.cu_q, full.kv_lens, full.block_table))
        run = S.KvHeadShardedDecode(nvb, shard, batch=full.batch, block_size=full.block_size,
                                    table_stride=full.table_stride, num_blocks=full.num_blocks, max_k=max(lens),
                                    device=torch.device("cuda", rank))
        first = []
        for a in sets:  # eager, one at a time: each set's output, checked against the single-GPU decode
            got = run(*a).clone()
            torch.cuda.synchronize()
            first.append(got)
        errs = [float((f.float().cpu() - r).abs().max()) for f, r in zip(first, refs)]
        graphs = [run.capture(*a) for a in sets]
        hist = torch.empty((steps,) + tuple(first[0].shape), dtype=first[0].dtype, device="cuda")
        for i in range(steps):  # no host sync: each step's output copied on the stream right behind it
            hist[i].copy_(run.replay(graphs[i % 3]))
        torch.cuda.synchronize()
        bad = [i for i in range(steps) if not torch.equal(hist[i], first[i % 3])]
        del graphs
        dev_err = nvb.device_error()
        dist.barrier()
        run.close()
        dist.destroy_process_group()
        q.put((rank, errs, bad[:8], len(bad), dev_err))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e), [], -1, -1))


# Many graph-replayed steps with no host sync between them, cycling three
# input sets: the output set alternates with the epoch and the data with
# period 3, so a peer store that landed after its epoch flag would leave the
# step-before-last's values in the copy and show as a mismatch.
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_gather_two_ranks_every_step_complete():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_stress_worker, args=(r, 2, port, q, 600)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, errs, bad, nbad, dev_err in results:
        assert isinstance(errs, list) and max(errs) <= 2e-2, (rank, errs)
        assert dev_err == 0 and nbad == 0, (rank, nbad, bad, dev_err)
