"""Batch sharding: host logic on the CPU (gloo, world size 2) and the
single-process multi-GPU forward on the GPU. Rows never interact, so a
sharded forward must equal the unsharded one bit for bit (the reference's
chunked-vs-unchunked check, src/run_case14.py:194-205)."""

from __future__ import annotations

import os

import pytest
import torch
import torch.multiprocessing as mp

import sharded


@pytest.mark.parametrize("batch,world", [(256, 8), (8, 8), (10, 4), (3, 8), (1, 2), (32, 3)])
def test_shard_bounds_partition_the_batch(batch, world):
    bounds = [sharded.shard_bounds(batch, world, r) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == batch
    for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in bounds]
    assert max(sizes) - min(sizes) <= 1


def _gloo_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # each rank's "device time" differs; the job time is the maximum
        t = sharded.max_over_ranks(1.5 + rank)
        b0, b1 = sharded.shard_bounds(256, world, rank)
        total = torch.tensor([b1 - b0])
        dist.all_reduce(total)
        q.put((rank, t, int(total.item())))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_gloo_world_size_2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_gloo_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = sorted(q.get(timeout=10) for _ in range(2))
    assert [t for _, t, _ in results] == [2.5, 2.5]
    assert all(total == 256 for _, _, total in results)


def test_max_over_ranks_without_process_group():
    assert sharded.max_over_ranks(3.25) == 3.25


@pytest.mark.gpu
@pytest.mark.parametrize("padding", [0.0, 0.3], ids=["dense", "padded"])
@pytest.mark.parametrize("mode", ["one_gpu_two_replicas", "all_gpus"])
def test_sharded_forward_matches_single_gpu(cuda_device, mode, padding):
    import optimized
    from oracle import StackConfig, generate_random_case, init_params

    n = torch.cuda.device_count()
    if mode == "all_gpus" and n < 2:
        pytest.skip("needs at least 2 GPUs")
    devices = ["cuda:0", "cuda:0"] if mode == "one_gpu_two_replicas" else [f"cuda:{i}" for i in range(n)]
    cfg = StackConfig(9, 128, 256, 4, 512, 2, True)
    params = init_params(cfg, seed=0)
    model = optimized.OptimizedTransformer(cfg)
    model.load_state_dict(params, strict=True)
    model = model.cuda().eval()
    shard = sharded.ShardedTransformer(model, devices)
    x, mask = generate_random_case(cfg, 21, padding_ratio=padding)
    xd, md = x.cuda(), mask.cuda()
    x2, _ = generate_random_case(cfg, 22)
    x2d = x2.cuda()
    with torch.inference_mode():
        want = model(xd, md).clone()
        want2 = model(x2d, md).clone()
        for _ in range(12):  # past graph capture in every replica; a new mask object every call
            got = shard(xd, md.clone()).clone()
        got2 = shard(x2d, md.clone()).clone()  # replays the captured graphs on new input
        got_again = shard(xd, md.clone()).clone()
        torch.cuda.synchronize()
    torch.testing.assert_close(got, want, atol=0, rtol=0)
    torch.testing.assert_close(got2, want2, atol=0, rtol=0)
    torch.testing.assert_close(got_again, want, atol=0, rtol=0)


# ---- the torchrun batch split (distributed.BatchSplitForward) --------------

@pytest.mark.parametrize("batch,world,micro", [(256, 8, 2), (8, 8, 2), (32, 8, 4), (10, 4, 3), (3, 4, 2), (32, 2, 16)])
def test_split_plan_partitions_the_batch(batch, world, micro):
    import distributed

    pieces = [p for r in range(world) for p in distributed.split_plan(batch, world, r, micro)]
    assert sorted(pieces) == pieces  # rank order, no overlap
    covered = [i for s, e in pieces for i in range(s, e)]
    assert covered == list(range(batch))
    assert all(e > s for s, e in pieces)
    for r in range(world):
        assert len(distributed.split_plan(batch, world, r, micro)) <= micro


def _gloo_plan_worker(rank, world, port, q):
    import torch.distributed as dist

    import distributed

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = distributed.split_plan(256, world, rank, 2)
        rows = torch.zeros(256, dtype=torch.int64)
        for s, e in mine:
            rows[s:e] += 1
        dist.all_reduce(rows)  # every sequence computed by exactly one rank
        box = [None] * world
        dist.all_gather_object(box, mine)
        q.put((rank, int(rows.min()), int(rows.max()), box))
    finally:
        dist.destroy_process_group()


def test_split_plan_gloo_world_size_2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 30500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_gloo_plan_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = sorted((q.get(timeout=10) for _ in range(2)), key=lambda t: t[0])
    for _, lo, hi, box in results:
        assert (lo, hi) == (1, 1)
        assert box == [[(0, 64), (64, 128)], [(128, 192), (192, 256)]]


def _ipc_owner(q_handle, q_done, result):
    import torch

    import _tklib as tk

    torch.cuda.set_device(0)
    src = torch.arange(6 * 1024, dtype=torch.float32, device="cuda").view(6, 1024)
    dst = torch.full((6, 1024), -1.0, device="cuda")
    torch.cuda.synchronize()
    q_handle.put((tk.peer_export(src), tk.peer_export(dst[1:])))  # an interior pointer: offset > 0
    assert q_done.get(timeout=120) == "written"
    torch.cuda.synchronize()
    want = torch.full((6, 1024), -1.0, device="cuda")
    want[1:] = src[[4, 5, 2, 3, 0]]  # the rows the peer gathered, written back from dst row 1 on
    result.put(bool(torch.equal(dst, want)))


def _ipc_peer(q_handle, q_done, result):
    import torch

    import _tklib as tk

    torch.cuda.set_device(0)
    (h_src, o_src), (h_dst, o_dst) = q_handle.get(timeout=120)
    assert o_src == 0 or o_src > 0
    src = tk.peer_import(h_src, o_src)
    dst = tk.peer_import(h_dst, o_dst)
    mine = torch.empty(5, 1024, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rb = 1024 * 4
    # gather rows 4,5 then 2,3 then 0 of the owner's tensor, then write them back strided
    tk.copy_rows(mine.data_ptr(), rb, src + 4 * rb, rb, rb, 2, stream)
    tk.copy_rows(mine.data_ptr() + 2 * rb, rb, src + 2 * rb, rb, rb, 2, stream)
    tk.copy_rows(mine.data_ptr() + 4 * rb, rb, src, rb, rb, 1, stream)
    tk.copy_rows(dst, rb, mine.data_ptr(), rb, rb, 5, stream)
    torch.cuda.synchronize()
    ok = bool(torch.equal(mine[0], torch.arange(4 * 1024, 5 * 1024, dtype=torch.float32, device="cuda")))
    tk.peer_release(src)
    tk.peer_release(dst)
    q_done.put("written")
    result.put(ok)


@pytest.mark.gpu
def test_peer_export_import_copy_rows_between_processes(cuda_device):
    """tk_peer_export / tk_peer_import / tk_copy_rows between two processes
    (one GPU is enough: CUDA IPC maps the owner's allocation into the peer;
    the processes order themselves on the host, no kernel waits on another)."""
    ctx = mp.get_context("spawn")
    q_handle, q_done, result = ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_ipc_owner, args=(q_handle, q_done, result)),
             ctx.Process(target=_ipc_peer, args=(q_handle, q_done, result))]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        assert p.exitcode == 0
    assert [result.get(timeout=10), result.get(timeout=10)] == [True, True]


def _free_port():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.gpu
@pytest.mark.parametrize("micro", [1, 3])
def test_batch_split_one_rank_matches_single_gpu(cuda_device, micro):
    """BatchSplitForward with a one-rank process group: the home buffers,
    the micro-batched copy-in / forward / copy-out pipeline (graph replays
    from the second step on) and the fences, against the one-GPU forward bit
    for bit. (Several ranks need one GPU each; their peer mappings are
    covered by the two-process IPC test.)"""
    import torch.distributed as dist

    import distributed
    import optimized
    from oracle import StackConfig, generate_random_case, init_params

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=cuda_device)
    try:
        cfg = StackConfig(7, 128, 256, 4, 512, 2, True)
        model = optimized.OptimizedTransformer(cfg)
        model.load_state_dict(init_params(cfg, seed=0), strict=True)
        model = model.cuda().eval()
        split = distributed.BatchSplitForward(model, (7, 128, 256), micro_batches=micro)
        x, _ = generate_random_case(cfg, 31)
        with torch.inference_mode():
            want = model(x.cuda()).clone()
            split.input.copy_(x)
            for _ in range(4):
                got = split.step()
            torch.cuda.synchronize()
            torch.testing.assert_close(got, want, atol=0, rtol=0)
            x2, _ = generate_random_case(cfg, 32)
            split.input.copy_(x2)
            got2 = split.step().clone()
            want2 = model(x2.cuda())
            torch.cuda.synchronize()
            torch.testing.assert_close(got2, want2, atol=0, rtol=0)
        split.close()
        with pytest.raises(Exception):
            split.step()
    finally:
        dist.destroy_process_group()
