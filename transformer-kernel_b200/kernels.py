"""Attention forward on the B200 kernel.

Same contract as the reference's ``src/kernels.py`` ``flash_attention``
(:250-294) and ``attention_supported`` (:96-103): ``q``/``k``/``v`` are
logically ``[B, H, S, hd]`` fp16 with arbitrary strides and a contiguous
last dimension (e.g. views straight out of the fused ``[B, S, 3, H, hd]``
QKV projection); the result is the context written directly as
``[B, S, H*hd]``. Scores are scaled after ``q.k`` (the baseline's order),
softmax statistics are fp32. Backed by ``tk_attn_fwd`` of libtk_b200; no
SDPA fallback.
"""

from __future__ import annotations

from typing import Optional

import torch

import _tklib as tk

__all__ = ["kernels_available", "attention_supported", "flash_attention"]


def kernels_available() -> bool:
    try:
        tk.lib()
        return True
    except tk.TKError:
        return False


def attention_supported(head_dim: int, dtype: torch.dtype, device: torch.device) -> bool:
    return (
        device.type == "cuda"
        and dtype == torch.float16
        and bool(tk.lib().tk_attn_supported(int(head_dim)))
    )


def flash_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float,
    causal: bool,
    kv_len: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Exact attention; returns the context in ``[B, S, H*hd]`` fp16.

    ``kv_len`` (int32 ``[B]``, optional) masks keys ``>= kv_len[b]`` -- the
    harness's prefix key-padding mask."""
    if not (q.shape == k.shape == v.shape) or q.dim() != 4:
        raise ValueError(f"q/k/v must share a [B, H, S, hd] shape, got {q.shape}, {k.shape}, {v.shape}")
    if not (q.dtype == k.dtype == v.dtype == torch.float16):
        raise tk.TKError("flash_attention", -2, "q/k/v must be float16")
    if not (q.stride() == k.stride() == v.stride()) or q.stride(-1) != 1:
        raise tk.TKError("flash_attention", -1, "q/k/v need identical strides and a contiguous last dimension")
    dev = tk.require_cuda(q, k, v, kv_len, out)
    B, H, S, hd = q.shape
    if out is None:
        out = torch.empty((B, S, H * hd), dtype=torch.float16, device=dev)
    elif out.shape != (B, S, H * hd) or out.stride(-1) != 1 or out.stride(0) != S * out.stride(1):
        raise ValueError("out must be [B, S, H*hd] with unit last stride and rows S*ld apart per batch")
    if kv_len is not None:
        kv_len = kv_len.to(dtype=torch.int32).contiguous()
    with torch.cuda.device(dev):
        tk.call(
            "tk_attn_fwd",
            q.data_ptr(), k.data_ptr(), v.data_ptr(),
            q.stride(0), q.stride(1), q.stride(2),
            out.data_ptr(), out.stride(1),
            B, S, H, hd, float(scale), int(bool(causal)),
            tk.ptr(kv_len), tk.stream_handle(dev),
        )
    return out
