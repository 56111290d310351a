"""One forward of a batch held on one GPU, split by batch over the GPUs of a node.

The north-star multi-GPU form of the layer-stack forward: one process per
GPU (torchrun), the whole ``[B, S, d]`` fp32 batch in the first rank's
device memory (the harness hands its input over on one device), every rank
computing the forward of its own shard of sequences, and the fp32 output
gathered back into the first rank's memory. Batch rows never interact
(``src/torch_transformer_benchmark.py:85-172`` has no cross-batch op), so
the only data exchange is that scatter and that gather -- the reference
runs the same split serially, one batch chunk after another on one device
(``src/run_case14.py:153-158``).

How the exchange runs on B200:

* The first rank's input and output buffers are mapped into every other
  rank's process (CUDA IPC, ``tk_peer_export`` / ``tk_peer_import``), so a
  shard moves as one strided copy (``tk_copy_rows``) that the copy engines
  carry over NVLink / NVSwitch without occupying an SM.
* Each rank cuts its shard into micro-batches and runs three streams: the
  copy-in of micro-batch j+1 and the copy-out of micro-batch j-1 overlap
  the forward of micro-batch j (graph-replayed), so most of the scatter and
  gather hides under the compute.
* Ordering across processes stays on the device: a one-element NCCL
  all-reduce on every rank's current stream opens a step (the first rank's
  writes of the input precede it) and one closes it (every rank's copy-out
  precedes it), so on the first rank the output is complete once its
  current stream passes the end of ``step()`` -- no host synchronisation.

Dense (all-valid) batches only; padded prefix masks run through
``OptimizedTransformer`` / ``ShardedTransformer``.
"""

from __future__ import annotations

from typing import List, Optional, Sequence

import torch

import _tklib as tk
import optimized
from sharded import shard_bounds

__all__ = ["BatchSplitForward", "split_plan"]


def split_plan(batch: int, world: int, rank: int, micro_batches: int) -> List[tuple]:
    """[start, stop) sequence ranges of `rank`'s micro-batches: its shard of
    the batch (``shard_bounds``) cut into at most `micro_batches` near-equal
    pieces. Over all ranks the pieces partition ``range(batch)``."""
    b0, b1 = shard_bounds(batch, world, rank)
    nb = b1 - b0
    if nb == 0:
        return []
    m = max(1, min(int(micro_batches), nb))
    return [(b0 + nb * i // m, b0 + nb * (i + 1) // m) for i in range(m)]


class BatchSplitForward:
    """``BatchSplitForward(model, shape, micro_batches=2, home=0, group=None)``
    on every rank of a process group (one process per GPU of one node).

    ``model`` is this rank's loaded ``OptimizedTransformer`` on its GPU (the
    same weights on every rank). On the home rank, ``input`` is the
    ``[B, S, d]`` fp32 batch buffer to fill and ``output`` the buffer that
    holds the result after ``step()``; both are ``None`` elsewhere. ``step()``
    is collective: every rank calls it once per forward.
    """

    def __init__(self, model: optimized.OptimizedTransformer, shape: Sequence[int], micro_batches: int = 2,
                 home: int = 0, group=None) -> None:
        import torch.distributed as dist

        if not dist.is_initialized():
            raise tk.TKError("BatchSplitForward", -1, "needs an initialised torch.distributed process group")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.home = home
        self.model = model
        self.device = model.layers[0].attention.q_proj.weight.device
        if self.device.type != "cuda":
            raise tk.TKError("BatchSplitForward", -1, "the model must live on this rank's CUDA device")
        B, S, d = (int(v) for v in shape)
        if d != model.d_model:
            raise ValueError(f"shape {tuple(shape)} does not match d_model {model.d_model}")
        self.shape = (B, S, d)
        self.row_bytes = S * d * 4  # one sequence of fp32 rows
        self.bounds = shard_bounds(B, self.world, self.rank)
        dev = self.device

        # home buffers, exported to the other ranks
        self.input: Optional[torch.Tensor] = None
        self.output: Optional[torch.Tensor] = None
        handles = None
        if self.rank == home:
            self.input = torch.empty(self.shape, dtype=torch.float32, device=dev)
            self.output = torch.empty(self.shape, dtype=torch.float32, device=dev)
            handles = [tk.peer_export(self.input), tk.peer_export(self.output)]
        box = [handles]
        dist.broadcast_object_list(box, src=home, group=group, device=dev)
        self._imported: List[int] = []
        if self.rank == home:
            self._in_base, self._out_base = self.input.data_ptr(), self.output.data_ptr()
        else:
            (hin, oin), (hout, oout) = box[0]
            self._in_base = tk.peer_import(hin, oin)
            self._imported.append(self._in_base)
            self._out_base = tk.peer_import(hout, oout)
            self._imported.append(self._out_base)

        # micro-batches of this rank's shard, two slots of device buffers
        self.micro = split_plan(B, self.world, self.rank, micro_batches)
        cb = max((e - s for s, e in self.micro), default=0)
        weights = model._weights()
        ffn = weights[0].ffn_in_w.shape[0]
        self.slots = []
        if cb:
            with torch.cuda.device(dev):
                for _ in range(2):
                    self.slots.append({
                        "x": torch.empty((cb, S, d), dtype=torch.float32, device=dev),
                        "out": torch.empty((cb, S, d), dtype=torch.float32, device=dev),
                        "bufs": model._activations(cb, S, d, ffn, dev), "graphs": {},
                        "in_ready": torch.cuda.Event(), "computed": torch.cuda.Event(),
                        "out_free": torch.cuda.Event()})
        self.cin = torch.cuda.Stream(dev)
        self.comp = torch.cuda.Stream(dev)
        self.cout = torch.cuda.Stream(dev)
        self._token = torch.zeros(1, dtype=torch.float32, device=dev)
        self._closed = False

    def _fence(self) -> None:
        """Stream-ordered rendezvous of all ranks (tiny NCCL all-reduce on the
        current stream; the host does not wait)."""
        import torch.distributed as dist

        dist.all_reduce(self._token, group=self.group)

    def step(self) -> Optional[torch.Tensor]:
        """This rank's share of one forward. Returns ``output`` on the home
        rank (complete once the current stream passes this point), else None."""
        if self._closed:
            raise tk.TKError("BatchSplitForward.step", -1, "called after close(): the peer buffers are unmapped")
        dev = self.device
        cur = torch.cuda.current_stream(dev)
        weights = self.model._weights()
        self._fence()  # the home rank's input is written
        start = torch.cuda.Event()
        start.record(cur)
        self.cin.wait_event(start)
        self.comp.wait_event(start)
        _, S, d = self.shape
        rb = self.row_bytes
        with torch.cuda.device(dev):
            for j, (s0, s1) in enumerate(self.micro):
                n = s1 - s0
                slot = self.slots[j % 2]
                xs, os_ = slot["x"][:n], slot["out"][:n]
                with torch.cuda.stream(self.cin):
                    self.cin.wait_event(slot["computed"])  # the forward that last read this slot is done
                    tk.copy_rows(xs.data_ptr(), rb, self._in_base + s0 * rb, rb, rb, n, self.cin.cuda_stream)
                    slot["in_ready"].record(self.cin)
                self.comp.wait_event(slot["in_ready"])
                self.comp.wait_event(slot["out_free"])  # the copy-out that last read this slot is done
                with torch.cuda.stream(self.comp):
                    self.model._slot_forward(slot, xs, os_, None, weights)
                slot["computed"].record(self.comp)
                with torch.cuda.stream(self.cout):
                    self.cout.wait_event(slot["computed"])
                    tk.copy_rows(self._out_base + s0 * rb, rb, os_.data_ptr(), rb, rb, n, self.cout.cuda_stream)
                    slot["out_free"].record(self.cout)
        cur.wait_stream(self.cin)
        cur.wait_stream(self.cout)
        self._fence()  # every rank's output rows have landed
        return self.output

    def close(self) -> None:
        """Unmap the home rank's buffers. Collective: every rank calls it
        before the process group is destroyed, and the home rank's buffers
        stay allocated until every other rank has unmapped them."""
        import torch.distributed as dist

        torch.cuda.synchronize(self.device)
        for ptr in self._imported:
            tk.peer_release(ptr)
        self._imported = []
        self._closed = True
        dist.barrier(group=self.group, device_ids=[self.device.index])
