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
