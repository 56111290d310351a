"""Whole-forward CUDA graph replay of the B200 forward.

Same policy as the reference's ``src/cuda_graphs.py`` ``GraphedTransformer``
(:61-164): the first ``WARMUP_BEFORE_CAPTURE`` calls per (shape, dtype,
device, mask lengths) run eagerly, then the forward is captured once on a
side-stream-warmed stream and every later call replays it. The kernels are
launched through ctypes on torch's current stream, so stream capture records
them like any other launch; their tensor maps are kernel parameters and are
baked into the graph.

What differs from the reference, and why:

* The caller's input is never a captured buffer. The forward's first launch
  (layer 0's LayerNorm, which also copies x into the forward's own fp32
  residual stream) runs eagerly on every call and reads whatever tensor the
  caller passes; the graph holds everything after it. So a call with a new
  input tensor costs no copy, and the caller's tensors are never written.
* The graph state keeps the prefix-length tensor it was captured with (the
  graph reads it by address on every replay).
* The returned tensor is the graph's output buffer: the next call on the
  same shape overwrites it (the reference returns its static output the same
  way). Clone it to keep it.
* Shapes that run as one launch (the small-shape whole-stack kernel) are not
  captured: the graph would hold that same single launch.
* A capture failure is raised, not turned into an eager fallback.
"""

from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from optimized import OptimizedTransformer, _outside_compile

__all__ = ["GraphedTransformer", "WARMUP_BEFORE_CAPTURE"]

WARMUP_BEFORE_CAPTURE = 8


class _GraphState:
    __slots__ = ("eager_calls", "graph", "static_out", "buffers", "lengths")

    def __init__(self) -> None:
        self.eager_calls = 0
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.static_out: Optional[torch.Tensor] = None
        self.buffers = None  # activation buffers the graph's kernels use
        self.lengths: Optional[torch.Tensor] = None  # prefix lengths the graph reads


class GraphedTransformer(OptimizedTransformer):
    """OptimizedTransformer whose forward replays as one CUDA graph."""

    def __init__(self, config, settings=None) -> None:
        super().__init__(config, settings)
        self._graph_states: Dict[Tuple, _GraphState] = {}

    def _apply(self, *args, **kwargs):
        result = super()._apply(*args, **kwargs)
        self._graph_states = {}
        return result

    def _load_from_state_dict(self, *args, **kwargs):
        # the captured graphs read the weight copies that a load rebuilds
        self._graph_states = {}
        return super()._load_from_state_dict(*args, **kwargs)

    @_outside_compile
    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        self._check_input(x)
        lengths, lkey = self._prefix_lengths_keyed(valid_token_mask)
        return self._finish(x, self._forward_lengths(x, lengths, lkey))

    def _forward_lengths(self, x: torch.Tensor, lengths: Optional[torch.Tensor], lkey) -> torch.Tensor:
        """Forward with the prefix lengths already resolved (``lkey`` is a
        hashable key of their values, None when dense)."""
        if self._uses_small_stack(x):
            return self._run(x, lengths)
        key = (tuple(x.shape), x.device, lkey)
        state = self._graph_states.setdefault(key, _GraphState())
        if state.graph is None:
            state.eager_calls += 1
            if state.eager_calls <= WARMUP_BEFORE_CAPTURE:
                return self._run(x, lengths)
            self._capture(state, x, lengths)
        with torch.cuda.device(x.device):
            self._head(x, state.buffers, self._weights())
        state.graph.replay()
        return state.static_out

    def _capture(self, state: _GraphState, x: torch.Tensor, lengths: Optional[torch.Tensor]) -> None:
        dev = x.device
        B, S, d = x.shape
        weights = self._weights()
        # Buffers are allocated before capture: nothing is allocated while the
        # stream captures (with peer access enabled between GPUs, a device
        # allocation is not permitted during capture).
        bufs = self._activations(B, S, d, weights[0].ffn_in_w.shape[0], dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.device(dev), torch.cuda.stream(side):
            for _ in range(2):
                self._head(x, bufs, weights)
                self._body(B, S, lengths, bufs, weights)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        # capture on a stream of x's device (torch's default capture stream
        # belongs to whichever device first captured)
        with torch.cuda.device(dev), torch.cuda.graph(graph, stream=torch.cuda.Stream(device=dev)):
            out = self._body(B, S, lengths, bufs, weights)
        state.static_out, state.buffers, state.lengths, state.graph = out, bufs, lengths, graph
