"""Drop-in ``UserOptimizedTransformer`` running on the B200 kernels.

Mirrors the reference's ``src/optimized.py`` surface: ``OptimizerSettings``,
``configure(**kw)`` / ``active_settings()`` (module-global settings, because
the harness constructs ``UserOptimizedTransformer(config)`` with no other
argument, :145-153) and ``OptimizedTransformer(config, settings=None)``
with the harness's ``forward(x, valid_token_mask=None)``.

The module tree is the harness's ``BaselineTransformer`` tree
(``src/torch_transformer_benchmark.py:125-160``: ``layers.{i}.norm1``,
``layers.{i}.attention.{q,k,v,out}_proj``, ``layers.{i}.norm2``,
``layers.{i}.ffn_in``, ``layers.{i}.ffn_out``, ``final_norm``), so the
harness's strict ``load_state_dict`` copy works unchanged. Derived tensors
(fp16 weights, the concatenated QKV weight) are plain attributes, never
parameters or buffers, and are dropped on ``_apply`` (``.to()``), as the
reference does (:224-244).

Forward, per layer (``T = B*S`` token rows, fp32 residual stream):

  h, x = LN1(x), copy of x                        tk_layernorm        (layer 0 only)
  qkv  = h Wqkv^T + bqkv                          tk_gemm  BIAS       fp16 [T, 3d]
  ctx  = attention(q, k, v views of qkv)          tk_attn_fwd         fp16 [T, d]
  x, h = x + ctx Wo^T + bo,  LN2(.)               tk_gemm_resid_ln    (d in {64,128,256} or
                                                  d % 256 == 0 up to 4096), else
                                                  tk_gemm RESID + tk_layernorm
  u    = gelu(h W1^T + b1)                        tk_gemm  GELU       fp16 [T, ffn]
  x, h = x + u W2^T + b2,  next LN1 / final LN    as the O-projection

The final LayerNorm writes the fp32 output directly. There is no CPU,
SDPA, cuBLAS or Triton path: anything the kernels cannot do raises.
"""

from __future__ import annotations

import weakref
from dataclasses import dataclass, replace
from typing import List, Optional

import torch
import torch.nn as nn

import _tklib as tk
import kernels
import linear as tk_linear

__all__ = ["OptimizerSettings", "OptimizedTransformer", "TransformerConfig", "configure", "active_settings"]


@dataclass(frozen=True)
class TransformerConfig:
    """Same fields as the harness's ``TransformerConfig``
    (``src/torch_transformer_benchmark.py:29-56``); any object with these
    attributes is accepted by ``OptimizedTransformer``."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool


@dataclass(frozen=True)
class OptimizerSettings:
    """Knobs of the B200 forward. None of them selects another backend."""

    # Fuse residual add + LayerNorm into the O-projection / FFN-out GEMM
    # epilogue when d_model fits one tile row (64, 128 or 256).
    fused_ln_epilogue: bool = True
    # Also fuse it for rows wider than a tile (d_model % 256 == 0, up to
    # 4096: tk_gemm_resid_ln, per-row partial statistics across the CTA-pair
    # tiles). Off by default: on one B200 at 65,536 x 1024 rows it measured
    # 0.45 ms (O-projection, K 1024) and 0.62 ms (FFN-out, K 4096) against
    # 0.24 ms and 0.54 ms for the in-place GEMM (TMA reduce-add) followed by
    # tk_layernorm; the shape dispatch table can turn it on per shape.
    fused_wide_ln: bool = False
    # Skip the one device->host sync that checks whether the mask is all-True.
    assume_dense_mask: bool = False
    # Synchronise after every forward and raise if a kernel's bounded
    # device-side wait gave up (debugging aid; costs a sync per call).
    check_device_errors: bool = False
    # Run shapes the one-launch whole-stack kernel takes (d_model = ffn =
    # 128, 2 or 4 heads, seq_len <= 128, equal LayerNorm eps) through it
    # instead of the per-layer kernel sequence (the reference's shape
    # dispatch picks per-shape paths the same way, src/dispatch.py:95-172).
    fused_small_stack: bool = True


_ACTIVE = OptimizerSettings()


def configure(**kwargs) -> OptimizerSettings:
    """Set the settings used by ``OptimizedTransformer(config)``."""
    global _ACTIVE
    _ACTIVE = replace(_ACTIVE, **kwargs)
    return _ACTIVE


def active_settings() -> OptimizerSettings:
    return _ACTIVE


def _outside_compile(fn):
    disable = getattr(getattr(torch, "compiler", None), "disable", None)
    return disable(fn) if disable is not None else fn


class _Attention(nn.Module):
    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        if d_model % num_heads != 0:
            raise ValueError("d_model must be divisible by num_heads")
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)


class _Block(nn.Module):
    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = _Attention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)


@dataclass
class _LayerWeights:
    norm1_w: torch.Tensor
    norm1_b: torch.Tensor
    norm1_eps: float
    qkv_w: torch.Tensor     # fp16 [3d, d] = [Wq; Wk; Wv]
    qkv_b: torch.Tensor     # fp32 [3d]
    out_w: torch.Tensor     # fp16 [d, d]
    out_b: torch.Tensor
    norm2_w: torch.Tensor
    norm2_b: torch.Tensor
    norm2_eps: float
    ffn_in_w: torch.Tensor  # fp16 [ffn, d]
    ffn_in_b: torch.Tensor
    ffn_out_w: torch.Tensor  # fp16 [d, ffn]
    ffn_out_b: torch.Tensor


class OptimizedTransformer(nn.Module):
    """B200 drop-in for the harness's ``UserOptimizedTransformer``."""

    def __init__(self, config, settings: Optional[OptimizerSettings] = None) -> None:
        super().__init__()
        self.config = config
        self.settings = settings if settings is not None else _ACTIVE
        self.layers = nn.ModuleList(
            [_Block(config.d_model, config.num_heads, config.ffn_dim) for _ in range(config.num_layers)]
        )
        self.final_norm = nn.LayerNorm(config.d_model)
        self.d_model = config.d_model
        self.num_heads = config.num_heads
        self.head_dim = config.d_model // config.num_heads
        self.attn_scale = self.head_dim ** -0.5
        self._weight_cache: Optional[List[_LayerWeights]] = None
        self._weight_cache_key: Optional[tuple] = None
        self._mask_ref: Optional[weakref.ReferenceType] = None
        self._mask_lengths: Optional[torch.Tensor] = None  # None = dense
        self._mask_key: Optional[tuple] = None
        # Optional launch trace: a list that receives (name, start, end)
        # CUDA events around every kernel launch of the next forwards.
        self.launch_trace: Optional[list] = None

    # -- caches ---------------------------------------------------------------
    def _apply(self, *args, **kwargs):
        result = super()._apply(*args, **kwargs)
        self._weight_cache = None
        self._weight_cache_key = None
        return result

    def _load_from_state_dict(self, *args, **kwargs):
        # A state-dict load copies into the existing parameters in place, so
        # their storage (the cache key) does not change: drop the derived
        # copies here. The reference relies on the load happening before the
        # first forward (src/optimized.py:266-273); this also covers a reload
        # after it.
        self._weight_cache = None
        self._weight_cache_key = None
        return super()._load_from_state_dict(*args, **kwargs)

    @_outside_compile
    def _weights(self) -> List[_LayerWeights]:
        """Per-layer fp16 GEMM weights (QKV concatenated) and fp32 bias /
        LayerNorm vectors, built once per (device, dtype, storage) of the
        parameters and dropped by ``_apply`` and by state-dict loads."""
        ref = self.layers[0].attention.q_proj.weight
        key = (ref.device, ref.dtype, ref.data_ptr())
        if self._weight_cache is not None and self._weight_cache_key == key:
            return self._weight_cache
        import dispatch

        dispatch.ensure_applied()  # the measured GEMM tile table, once per process
        built = []
        with torch.no_grad():
            f16 = lambda t: t.detach().to(torch.float16).contiguous()  # noqa: E731
            f32 = lambda t: t.detach().to(torch.float32).contiguous()  # noqa: E731
            for layer in self.layers:
                a = layer.attention
                built.append(
                    _LayerWeights(
                        norm1_w=f32(layer.norm1.weight), norm1_b=f32(layer.norm1.bias), norm1_eps=layer.norm1.eps,
                        qkv_w=f16(torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0)),
                        qkv_b=f32(torch.cat([a.q_proj.bias, a.k_proj.bias, a.v_proj.bias], 0)),
                        out_w=f16(a.out_proj.weight), out_b=f32(a.out_proj.bias),
                        norm2_w=f32(layer.norm2.weight), norm2_b=f32(layer.norm2.bias), norm2_eps=layer.norm2.eps,
                        ffn_in_w=f16(layer.ffn_in.weight), ffn_in_b=f32(layer.ffn_in.bias),
                        ffn_out_w=f16(layer.ffn_out.weight), ffn_out_b=f32(layer.ffn_out.bias),
                    )
                )
        self._final = (f32(self.final_norm.weight), f32(self.final_norm.bias), self.final_norm.eps)
        self._small_pack = None  # packed weights of the one-launch small-shape kernel, built on first use
        self._weight_cache, self._weight_cache_key = built, key
        return built

    def _small_stack_pack(self, weights: List[_LayerWeights]):
        """(w fp16 [L*768, 128], vec fp32 [L, 1280], eps) for tk_stack_small,
        or None when the LayerNorm epsilons differ (the kernel takes one)."""
        if self._small_pack is not None:
            return self._small_pack
        eps = {w.norm1_eps for w in weights} | {w.norm2_eps for w in weights} | {self._final[2]}
        if len(eps) != 1:
            self._small_pack = False
            return None
        with torch.no_grad():
            w = torch.cat([torch.cat([lw.qkv_w, lw.out_w, lw.ffn_in_w, lw.ffn_out_w], 0) for lw in weights], 0)
            vec = torch.stack([torch.cat([lw.qkv_b, lw.out_b, lw.ffn_in_b, lw.ffn_out_b, lw.norm1_w, lw.norm1_b,
                                          lw.norm2_w, lw.norm2_b]) for lw in weights], 0)
        self._small_pack = (w.contiguous(), vec.contiguous(), float(eps.pop()))
        return self._small_pack

    @_outside_compile
    def _prefix_lengths(self, mask: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
        """``None`` for an all-True (or absent) mask, else the int32 per-row
        prefix lengths. One device->host sync per distinct mask object
        (weakref memo, like the reference's ``_mask_is_dense``, :362-389).
        Masks that are not per-row prefixes -- the only kind the harness's
        ``generate_random_case`` makes (:261-271) -- raise."""
        return self._prefix_lengths_keyed(mask)[0]

    def _prefix_lengths_keyed(self, mask: Optional[torch.Tensor]):
        """(lengths, key): ``_prefix_lengths`` plus a hashable key of the
        lengths' values (None when dense), taken at the same sync."""
        if mask is None or self.settings.assume_dense_mask:
            return None, None
        if self._mask_ref is not None and self._mask_ref() is mask:
            return self._mask_lengths, self._mask_key
        m = mask.to(torch.bool)
        lengths = m.sum(dim=-1, dtype=torch.int32)
        if bool(m.all()):
            result, key = None, None
        else:
            prefix = torch.arange(m.shape[-1], device=m.device)[None, :] < lengths[:, None]
            if not bool((prefix == m).all()):
                raise tk.TKError("forward", -2, "valid_token_mask must be a per-row prefix (True then False)")
            result = lengths.contiguous()
            key = tuple(result.tolist())
        self._mask_ref = weakref.ref(mask)
        self._mask_lengths, self._mask_key = result, key
        return result, key

    # -- forward --------------------------------------------------------------
    # The forward is opaque to torch.compile (the harness's --compile-user
    # wraps the model, src/torch_transformer_benchmark.py:586-591,703): it is
    # a sequence of library launches on raw pointers with nothing for dynamo
    # to trace, and its cached buffers must stay ordinary allocations
    # (src/optimized.py:64-77 keeps its cache builders out for that reason).
    @_outside_compile
    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        self._check_input(x)
        lengths = self._prefix_lengths(valid_token_mask)
        return self._finish(x, self._run(x, lengths))

    def _check_input(self, x: torch.Tensor) -> None:
        if not x.is_cuda:
            raise tk.TKError("forward", -1, "OptimizedTransformer runs on the B200 kernels only; x must be a CUDA tensor")
        if x.dim() != 3 or x.shape[-1] != self.d_model:
            raise ValueError(f"expected x of shape [B, S, {self.d_model}], got {tuple(x.shape)}")

    def _finish(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Optional device-error check; the output in x's dtype (the
        reference casts back too, src/optimized.py:408)."""
        if self.settings.check_device_errors:
            tk.check_device_errors(x.device)
        return out if out.dtype == x.dtype else out.to(x.dtype)

    def _activations(self, B: int, S: int, d: int, ffn: int, dev: torch.device):
        """Activation buffers of one forward: residual stream fp32 [T, d], h
        fp16 [T, d], qkv fp16 [T, 3d], ctx fp16 [B, S, d], u fp16 [T, ffn],
        the output fp32 [T, d], and the (zeroed) workspace of the residual +
        LayerNorm GEMMs for rows wider than a tile, from the caching
        allocator. A workspace sized for T rows serves any shorter forward."""
        T = B * S
        ws = max(256, tk_linear.ln_workspace_bytes(T, d))
        return (torch.empty((T, d), dtype=torch.float32, device=dev),
                torch.empty((T, d), dtype=torch.float16, device=dev),
                torch.empty((T, 3 * d), dtype=torch.float16, device=dev),
                torch.empty((B, S, d), dtype=torch.float16, device=dev),
                torch.empty((T, ffn), dtype=torch.float16, device=dev),
                torch.empty((T, d), dtype=torch.float32, device=dev),
                torch.zeros(ws, dtype=torch.uint8, device=dev))

    def _uses_small_stack(self, x: torch.Tensor) -> bool:
        """Whether a forward over x runs as one tk_stack_small launch."""
        B, S, d = x.shape
        ffn = self.layers[0].ffn_in.weight.shape[0]
        if not (self.settings.fused_small_stack and tk.lib().tk_stack_small_supported(d, self.num_heads, ffn, S)):
            return False
        return bool(self._small_stack_pack(self._weights()))

    def _small_stack(self, x, lengths, out, weights) -> Optional[torch.Tensor]:
        """The whole forward in one tk_stack_small launch when the shape and
        settings allow it; None otherwise."""
        B, S, d = x.shape
        if not self._uses_small_stack(x):
            return None
        ffn = weights[0].ffn_in_w.shape[0]
        w, vec, eps = self._small_stack_pack(weights)
        xin = x if (x.dtype == torch.float32 and x.is_contiguous()) else x.to(torch.float32).contiguous()
        if out is None:
            out = torch.empty((B, S, d), dtype=torch.float32, device=x.device)
        fg, fb, _ = self._final
        self._launch("stack_small", lambda: tk.call(
            "tk_stack_small", xin.data_ptr(), out.data_ptr(), w.data_ptr(), vec.data_ptr(), fg.data_ptr(),
            fb.data_ptr(), eps, tk.ptr(lengths), B, S, d, self.num_heads, ffn, len(weights),
            1 if self.config.causal else 0, self.attn_scale, tk.stream_handle(x.device)))
        return out.view(B, S, d)

    def _launch(self, name, fn, *args, **kwargs):
        """Run one library call; with ``launch_trace`` set, bracket it with
        CUDA events on the current stream."""
        trace = self.launch_trace
        if trace is None:
            return fn(*args, **kwargs)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        result = fn(*args, **kwargs)
        end.record()
        trace.append((name, start, end))
        return result

    def _layer_norm(self, src, w, b, eps, dst, lengths=None, seq=0, copy_to=None):
        """dst = LN(src) over fp32 rows; rows past their prefix length are
        zeroed when ``lengths`` is given; ``copy_to`` also receives src."""
        T, d = src.shape
        tk.call(
            "tk_layernorm",
            src.data_ptr(), tk.TK_F32, src.stride(0), None, 0, 0,
            tk.ptr(copy_to), 0 if copy_to is None else copy_to.stride(0),
            w.data_ptr(), b.data_ptr(), float(eps),
            dst.data_ptr(), tk.dtype_code(dst.dtype), dst.stride(0),
            tk.ptr(lengths), seq, T, d, tk.stream_handle(src.device),
        )

    def _head(self, x: torch.Tensor, bufs, weights: List[_LayerWeights]) -> None:
        """First launch of the per-layer forward: h = LN1(x), and the fp32
        residual stream starts as a copy of x in its own buffer. Only this
        launch reads the caller's x, so everything after it (``_body``)
        touches the forward's own buffers alone -- which is what a captured
        graph replays."""
        B, S, d = x.shape
        xin = x.reshape(B * S, d)
        if xin.dtype != torch.float32 or xin.stride(-1) != 1 or xin.stride(0) != d:
            xin = xin.to(torch.float32).contiguous()
        res, h = bufs[0], bufs[1]
        w0 = weights[0]
        self._launch("ln_in", self._layer_norm, xin, w0.norm1_w, w0.norm1_b, w0.norm1_eps, h, copy_to=res)

    def _body(self, B: int, S: int, lengths: Optional[torch.Tensor], bufs, weights: List[_LayerWeights],
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Every launch after ``_head``: the layers (the residual stream is
        updated in place) and the final LayerNorm into ``out`` (default the
        forward's own output buffer). Returns the output as [B, S, d]."""
        res, h, qkv, ctx, u, out_ws, ln_ws = bufs
        T, d = res.shape
        ffn = u.shape[1]
        hd = self.head_dim
        fused = self.settings.fused_ln_epilogue and tk_linear.fused_ln_supported(d) and (
            d in (64, 128, 256) or self.settings.fused_wide_ln)
        seq = S if lengths is not None else 0
        out = out_ws if out is None else out.view(T, d)
        run, lin = self._launch, tk_linear.linear
        # q/k/v as [B, H, S, hd] views of the fused projection
        qkv4 = qkv.view(B, S, 3, self.num_heads, hd)
        q, k, v = qkv4.permute(2, 0, 3, 1, 4).unbind(0)
        last = len(weights) - 1
        for i, w in enumerate(weights):
            run("gemm_qkv", lin, h, w.qkv_w, w.qkv_b, "bias", out=qkv)
            run("attn", kernels.flash_attention, q, k, v, self.attn_scale, self.config.causal,
                kv_len=lengths, out=ctx)
            ctx2 = ctx.view(T, d)
            if fused:
                run("gemm_o_ln", lin, ctx2, w.out_w, w.out_b, "resid_ln", resid=res, sum_out=res,
                    ln_weight=w.norm2_w, ln_bias=w.norm2_b, eps=w.norm2_eps, out=h, workspace=ln_ws)
            else:
                run("gemm_o", lin, ctx2, w.out_w, w.out_b, "resid", resid=res, sum_out=res)
                run("ln", self._layer_norm, res, w.norm2_w, w.norm2_b, w.norm2_eps, h)
            run("gemm_ffn_in", lin, h, w.ffn_in_w, w.ffn_in_b, "gelu", out=u)
            if i < last:
                nw, nb, neps, dst = weights[i + 1].norm1_w, weights[i + 1].norm1_b, weights[i + 1].norm1_eps, h
            else:
                nw, nb, neps = self._final
                dst = out
            if fused:
                run("gemm_ffn_out_ln", lin, u, w.ffn_out_w, w.ffn_out_b, "resid_ln", resid=res, sum_out=res,
                    ln_weight=nw, ln_bias=nb, eps=neps, out=dst, row_len=lengths, seq_len=seq, workspace=ln_ws)
            else:
                run("gemm_ffn_out", lin, u, w.ffn_out_w, w.ffn_out_b, "resid", resid=res, sum_out=res,
                    row_len=lengths, seq_len=seq)
                run("ln" if i < last else "ln_out", self._layer_norm, res, nw, nb, neps, dst, lengths, seq)
        return out.view(B, S, d)

    def _run(self, x: torch.Tensor, lengths: Optional[torch.Tensor], out: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, S, d = x.shape
        dev = x.device
        weights = self._weights()
        with torch.cuda.device(dev):
            fused = self._small_stack(x, lengths, out, weights)
            if fused is not None:
                return fused
            bufs = self._activations(B, S, d, weights[0].ffn_in_w.shape[0], dev)
            self._head(x, bufs, weights)
            return self._body(B, S, lengths, bufs, weights, out)

    # -- host-streamed forward --------------------------------------------------
    @_outside_compile
    def forward_from_host(
        self,
        x_host: torch.Tensor,
        valid_token_mask: Optional[torch.Tensor] = None,
        out_host: Optional[torch.Tensor] = None,
        chunks: int = 2,
        device: Optional[torch.device] = None,
    ) -> torch.Tensor:
        """Forward over a batch that lives in (pinned) host memory.

        The batch is cut into ``chunks`` slices of whole sequences (rows are
        independent, so slicing is exact). Three internal streams overlap the
        H2D copy of a slice, the forward of the one before it and the D2H copy
        of the one before that -- the copy engines and the SMs work at the
        same time, where the reference's out-of-core runner copies and
        computes in turn (``src/run_case14.py:286-298``). Two slots of device
        buffers alternate, also across calls, and each slot is guarded by its
        own events, so consecutive calls pipeline into one another: the next
        call's first copy and forward start while this call's last slice is
        still being copied back. Dense slices replay a CUDA graph captured per
        (slot, slice size).

        Returns ``out_host`` (fp32, pinned). It is complete once the current
        CUDA stream reaches the point where this call returned (synchronise
        before reading it on the host). The internal streams order themselves
        after the caller's stream only for the weight copies and prefix
        lengths this call builds; x_host is read asynchronously, so it must
        not be rewritten before the call's work has completed.
        """
        if x_host.is_cuda:
            raise ValueError("forward_from_host takes a host tensor; use forward() for device tensors")
        if x_host.dim() != 3 or x_host.shape[-1] != self.d_model:
            raise ValueError(f"expected x of shape [B, S, {self.d_model}], got {tuple(x_host.shape)}")
        dev = device or self.layers[0].attention.q_proj.weight.device
        if dev.type != "cuda":
            raise tk.TKError("forward_from_host", -1, "the model must live on a CUDA device")
        B, S, d = x_host.shape
        if x_host.dtype != torch.float32:
            x_host = x_host.float()
        if out_host is None:
            out_host = torch.empty((B, S, d), dtype=torch.float32, pin_memory=True)
        caller = torch.cuda.current_stream(dev)
        cache_before = self._weight_cache
        with torch.cuda.device(dev):
            weights = self._weights()
        lengths, _ = self._prefix_lengths_keyed(valid_token_mask)
        if lengths is not None:
            lengths = lengths.to(dev)
        n = max(1, min(int(chunks), B))
        bounds = [B * i // n for i in range(n + 1)]
        cb = max(bounds[i + 1] - bounds[i] for i in range(n))
        ctx = self._stream_context(dev, S, d, cb, weights)
        h2d, compute, d2h = ctx["h2d"], ctx["compute"], ctx["d2h"]
        if self._weight_cache is not cache_before or (lengths is not None and lengths is not ctx["lengths"]):
            # weight copies / lengths were just built on the caller's stream
            ready = torch.cuda.Event()
            ready.record(caller)
            compute.wait_event(ready)
            ctx["lengths"] = lengths
        with torch.cuda.device(dev):
            for i in range(n):
                s = ctx["next_slot"]
                ctx["next_slot"] ^= 1
                b0, b1 = bounds[i], bounds[i + 1]
                nb = b1 - b0
                slot = ctx["slots"][s]
                xs, os_ = slot["x"][:nb], slot["out"][:nb]
                with torch.cuda.stream(h2d):
                    h2d.wait_event(slot["computed"])   # the last forward that read this input slot is done
                    xs.copy_(x_host[b0:b1], non_blocking=True)
                    slot["in_ready"].record(h2d)
                compute.wait_event(slot["in_ready"])
                compute.wait_event(slot["out_free"])   # the last D2H that read this output slot is done
                with torch.cuda.stream(compute):
                    self._slot_forward(slot, xs, os_, None if lengths is None else lengths[b0:b1], weights)
                slot["computed"].record(compute)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(slot["computed"])
                    out_host[b0:b1].copy_(os_, non_blocking=True)
                    slot["out_free"].record(d2h)
            caller.wait_stream(d2h)
        if self.settings.check_device_errors:
            tk.check_device_errors(dev)
        return out_host

    def _stream_context(self, dev, S, d, cb, weights):
        """Streams, two slots of device buffers (input, output, activations)
        and their events for ``forward_from_host``; rebuilt when the slice
        shape changes."""
        key = (dev, S, d, cb)
        ctx = getattr(self, "_stream_ctx", None)
        if ctx is not None and ctx["key"] == key:
            return ctx
        if ctx is not None:
            # the old slots may still be read and written by work queued on the
            # old streams, which the caching allocator does not know about: let
            # it finish before the buffers go back to the allocator
            for name in ("h2d", "compute", "d2h"):
                ctx[name].synchronize()
            self._stream_ctx = None
        ffn = weights[0].ffn_in_w.shape[0]
        with torch.cuda.device(dev):
            slots = [{"x": torch.empty((cb, S, d), dtype=torch.float32, device=dev),
                      "out": torch.empty((cb, S, d), dtype=torch.float32, device=dev),
                      "bufs": self._activations(cb, S, d, ffn, dev),
                      "graphs": {},
                      "in_ready": torch.cuda.Event(), "computed": torch.cuda.Event(),
                      "out_free": torch.cuda.Event()} for _ in range(2)]
            ctx = {"key": key, "h2d": torch.cuda.Stream(dev), "compute": torch.cuda.Stream(dev),
                   "d2h": torch.cuda.Stream(dev), "slots": slots, "next_slot": 0, "lengths": None}
        self._stream_ctx = ctx
        return ctx

    def _slot_forward(self, slot, xs, os_, lengths, weights) -> None:
        """Forward of one slice on the current stream: slot buffers in, slot
        output out. Dense slices of the per-layer path replay a graph captured
        per slice size on the second use (everything they touch is the slot's
        own); padded slices and one-launch shapes run eagerly."""
        nb, S, d = xs.shape
        if lengths is not None or self._uses_small_stack(xs):
            self._run(xs, lengths, out=os_)
            return
        # views of the slot's buffers for nb sequences; the workspace (last)
        # serves any row count up to the one it was sized for
        bufs = tuple(b[:nb * S] if b.dim() == 2 else b[:nb] for b in slot["bufs"][:-1]) + (slot["bufs"][-1],)
        g = slot["graphs"].get(nb)
        if g is None:
            self._head(xs, bufs, weights)
            self._body(nb, S, None, bufs, weights, out=os_)
            slot["graphs"][nb] = "warm"
            return
        if g == "warm":
            graph = torch.cuda.CUDAGraph()
            # thread-local capture mode: other threads of the process (a
            # process group's watchdog) may query events meanwhile
            with torch.cuda.graph(graph, stream=torch.cuda.Stream(device=xs.device),
                                  capture_error_mode="thread_local"):
                self._head(xs, bufs, weights)
                self._body(nb, S, None, bufs, weights, out=os_)
            slot["graphs"][nb] = g = graph
        g.replay()
