"""Batch sharding of the layer-stack forward over the GPUs of one box.

Batch rows never interact in the stack (no cross-batch op anywhere in
``src/torch_transformer_benchmark.py:85-172``), so the forward partitions by
batch with no data-path collective; the reference relies on the same fact
for its chunked runner (``src/run_case14.py:14-16,153-158``). Two forms:

* ``ShardedTransformer`` -- one process drives N local GPUs: the input on
  the first device is split by batch, each shard is copied to its device
  over NVLink (copy engines, peer access), every device runs its own
  graph-replayed replica on its own stream, and the output shards are
  gathered back into one tensor on the first device. The first device's
  current stream waits on all of it, so CUDA events recorded there (the
  harness's timing, ``:487-500``) bracket the whole sharded forward.
* ``shard_bounds`` / ``max_over_ranks`` -- helpers for one-process-per-GPU
  runs under torchrun (``bench.py``): each rank takes its batch slice, and
  the job's time is the maximum over ranks.
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import torch

import _tklib as tk
import cuda_graphs
import optimized


def shard_bounds(batch: int, world: int, rank: int) -> tuple:
    """[start, stop) of `rank`'s batch rows when `batch` rows are split over
    `world` ranks as evenly as possible (the first `batch % world` ranks
    take one extra row)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(value: float, device: Optional[torch.device] = None, group=None) -> float:
    """Maximum of a per-rank scalar over the default process group (the
    job's time is its slowest rank's time). Works with NCCL (pass the rank's
    CUDA device) and gloo (CPU)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


class ShardedTransformer(torch.nn.Module):
    """Forward of one weight set over several local GPUs, sharded by batch.

    ``ShardedTransformer(model, devices)`` takes a loaded
    ``OptimizedTransformer`` (on ``devices[0]``) and builds graph-replayed
    replicas on the other devices (weights copied once). ``forward(x,
    valid_token_mask=None)`` takes ``x`` on ``devices[0]`` and returns the
    full ``[B, S, d]`` fp32 output there. The returned tensor is reused by
    the next call with the same shape (like ``GraphedTransformer``'s output);
    clone it to keep it. A device may be listed more than once (replicas on
    one GPU; used to test the split/gather logic on one GPU).
    """

    def __init__(self, model: optimized.OptimizedTransformer, devices: Sequence) -> None:
        super().__init__()
        devices = [torch.device(d) for d in devices]
        if not devices or any(d.type != "cuda" for d in devices):
            raise tk.TKError("ShardedTransformer", -1, "devices must be CUDA devices")
        self.devices: List[torch.device] = devices
        state = {k: v.detach() for k, v in model.state_dict().items()}
        self.replicas = []
        for dev in devices:
            rep = cuda_graphs.GraphedTransformer(model.config, model.settings)
            rep.load_state_dict({k: v.to(dev) for k, v in state.items()}, strict=True)
            self.replicas.append(rep.to(dev).eval())
        self.streams = [torch.cuda.Stream(device=d) for d in devices]
        # per-shard streams on the first device: a cross-device copy runs on
        # the source device's current stream, so each shard's scatter gets its
        # own stream there and the shards' copies run side by side
        self.home_streams = [torch.cuda.Stream(device=devices[0]) for _ in devices]
        self._bufs = {}
        self._lengths = {}  # (shard, lengths key) -> that shard's prefix lengths on its device
        self._mask_owner = self.replicas[0]  # its dense-mask memo (one sync per mask object)

    def _shard_buffers(self, x: torch.Tensor, bounds):
        key = (tuple(x.shape), x.dtype)
        bufs = self._bufs.get(key)
        if bufs is None:
            inputs = []
            for (b0, b1), dev in zip(bounds, self.devices):
                inputs.append(torch.empty((b1 - b0,) + tuple(x.shape[1:]), dtype=torch.float32, device=dev))
            out = torch.empty(x.shape, dtype=torch.float32, device=self.devices[0])
            bufs = (inputs, out)
            self._bufs = {key: bufs}
        return bufs

    def _shard_lengths(self, r: int, lengths: Optional[torch.Tensor], lkey, b0: int, b1: int):
        """Shard r's prefix lengths on its device, built once per distinct
        lengths from the host-side key by a blocking host-to-device copy, so
        no stream ordering is involved."""
        if lengths is None:
            return None, None
        key = (r, lkey)
        got = self._lengths.get(key)
        if got is None:
            if len(self._lengths) > 64:
                self._lengths.clear()
            got = (torch.tensor(lkey[b0:b1], dtype=torch.int32, device=self.devices[r]), lkey[b0:b1])
            self._lengths[key] = got
        return got

    @optimized._outside_compile
    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        home = self.devices[0]
        if x.device != home:
            raise ValueError(f"x must be on {home}")
        n = len(self.devices)
        B = x.shape[0]
        bounds = [shard_bounds(B, n, r) for r in range(n)]
        inputs, out = self._shard_buffers(x, bounds)
        lengths, lkey = self._mask_owner._prefix_lengths_keyed(valid_token_mask)
        main = torch.cuda.current_stream(home)
        ready = torch.cuda.Event()
        ready.record(main)
        done = []
        for r, (dev, stream) in enumerate(zip(self.devices, self.streams)):
            b0, b1 = bounds[r]
            if b1 == b0:
                continue
            xin = inputs[r]
            len_r, lkey_r = self._shard_lengths(r, lengths, lkey, b0, b1)
            hs = self.home_streams[r]
            hs.wait_event(ready)
            # Nested stream contexts make hs the first device's current stream
            # and `stream` the shard device's, so torch runs the scatter on hs
            # (source side) and the gather on `stream` (source side), and
            # makes the other side wait for each copy.
            with torch.cuda.stream(hs), torch.cuda.stream(stream):
                stream.wait_event(ready)
                xin.copy_(x[b0:b1], non_blocking=True)        # scatter (peer copy over NVLink)
                y = self.replicas[r]._forward_lengths(xin, len_r, lkey_r)
                out[b0:b1].copy_(y, non_blocking=True)        # gather onto the first device
                ev = torch.cuda.Event()
                ev.record(stream)
            done.append(ev)
        for ev in done:
            main.wait_event(ev)
        return out
