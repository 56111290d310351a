"""Fused LayerNorm / residual-add + LayerNorm on the B200 kernels.

Same names, arguments and return values as the reference's
``src/fused_kernels.py`` (``ln_fwd`` :164-193, ``add_ln_fwd`` :196-238,
``can_fuse`` :62-64, ``MAX_FUSED_SIZE`` :59), backed by ``tk_layernorm`` of
libtk_b200 (warp-per-row, 128-bit loads, fp32 two-pass statistics).
Unlike the reference there is no eager fallback: CPU tensors or widths the
kernel does not take raise ``TKError``.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

import _tklib as tk

MAX_FUSED_SIZE = 8192


def can_fuse(x: torch.Tensor) -> bool:
    """Whether the kernels apply to activations shaped like ``x``."""
    return x.is_cuda and bool(tk.lib().tk_layernorm_supported(x.shape[-1]))


def _rows(t: torch.Tensor) -> torch.Tensor:
    t2 = t.reshape(-1, t.shape[-1])
    return t2 if t2.stride(-1) == 1 else t2.contiguous()


def ln_fwd(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float,
    out_dtype: Optional[torch.dtype] = None,
) -> torch.Tensor:
    """LayerNorm over the last dim, fp32 statistics, output in ``out_dtype``."""
    out_dtype = x.dtype if out_dtype is None else out_dtype
    dev = tk.require_cuda(x, weight, bias)
    shape = x.shape
    x2 = _rows(x)
    out = torch.empty(x2.shape, dtype=out_dtype, device=dev)
    w, b = weight.float().contiguous(), bias.float().contiguous()
    with torch.cuda.device(dev):
        tk.call(
            "tk_layernorm",
            x2.data_ptr(), tk.dtype_code(x2.dtype), x2.stride(0),
            None, 0, 0, None, 0,
            w.data_ptr(), b.data_ptr(), float(eps),
            out.data_ptr(), tk.dtype_code(out_dtype), out.stride(0),
            None, 0, x2.shape[0], x2.shape[1], tk.stream_handle(dev),
        )
    return out.view(shape)


def add_ln_fwd(
    x: torch.Tensor,
    y: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float,
    out_dtype: Optional[torch.dtype] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Fused residual add + LayerNorm: returns ``(s, h)`` with
    ``s = x + y`` in ``x``'s dtype and ``h = LayerNorm(s)`` in ``out_dtype``;
    the add and the statistics are fp32."""
    if x.shape != y.shape:
        raise ValueError(f"shape mismatch: {x.shape} vs {y.shape}")
    out_dtype = x.dtype if out_dtype is None else out_dtype
    dev = tk.require_cuda(x, y, weight, bias)
    shape = x.shape
    x2, y2 = _rows(x), _rows(y)
    s = torch.empty(x2.shape, dtype=x.dtype, device=dev)
    h = torch.empty(x2.shape, dtype=out_dtype, device=dev)
    w, b = weight.float().contiguous(), bias.float().contiguous()
    with torch.cuda.device(dev):
        tk.call(
            "tk_layernorm",
            x2.data_ptr(), tk.dtype_code(x2.dtype), x2.stride(0),
            y2.data_ptr(), tk.dtype_code(y2.dtype), y2.stride(0),
            s.data_ptr(), s.stride(0),
            w.data_ptr(), b.data_ptr(), float(eps),
            h.data_ptr(), tk.dtype_code(out_dtype), h.stride(0),
            None, 0, x2.shape[0], x2.shape[1], tk.stream_handle(dev),
        )
    return s.view(shape), h.view(shape)
