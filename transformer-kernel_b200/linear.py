"""tcgen05 GEMM with fused epilogues (replaces ``F.linear`` on the hot path).

``linear(a, w, bias, epilogue=...)`` computes ``a @ w.T + bias`` on the
tensor cores with fp16 operands and fp32 accumulation (``tk_gemm``), and
fuses what follows the projection in the reference's forward
(``src/optimized.py:572,627,632-636``; ``src/fused_kernels.py:196-238``):

* ``"bias"``          -> fp16 ``a @ w.T + b``
* ``"gelu"``          -> fp16 ``gelu_erf(a @ w.T + b)`` (fp32 erf)
* ``"resid"``         -> fp32 ``s = resid + a @ w.T + b`` (written to ``sum_out``)
* ``"resid_ln"``      -> as ``"resid"``, and ``out = LayerNorm(s)`` with fp32
  statistics: ``N`` in {64, 128, 256} in one tile (``tk_gemm``), or
  ``N % 256 == 0`` up to 4096 with per-row partial statistics in a workspace
  (``tk_gemm_resid_ln``; pass ``workspace``, a zeroed uint8 tensor of
  ``ln_workspace_bytes(M, N)`` bytes, to reuse one across calls)

``w`` is the ``nn.Linear`` weight ``[N, K]`` in fp16 as-is. No fallback.
"""

from __future__ import annotations

from typing import Optional

import torch

import _tklib as tk

EPILOGUES = {
    "bias": tk.EPI_BIAS,
    "gelu": tk.EPI_BIAS_GELU,
    "resid": tk.EPI_BIAS_RESID,
    "resid_ln": tk.EPI_BIAS_RESID_LN,
}


def fused_ln_supported(n: int) -> bool:
    """Whether residual add + LayerNorm fuses into the GEMM for rows of n."""
    return bool(tk.lib().tk_gemm_resid_ln_supported(1, int(n), 8))


def ln_workspace_bytes(m: int, n: int) -> int:
    """Workspace bytes of a ``"resid_ln"`` GEMM with m rows of n columns (0
    when one tile holds the row)."""
    return int(tk.lib().tk_gemm_resid_ln_workspace_bytes(int(m), int(n)))


def linear(
    a: torch.Tensor,
    w: torch.Tensor,
    bias: torch.Tensor,
    epilogue: str = "bias",
    *,
    resid: Optional[torch.Tensor] = None,
    sum_out: Optional[torch.Tensor] = None,
    ln_weight: Optional[torch.Tensor] = None,
    ln_bias: Optional[torch.Tensor] = None,
    eps: float = 1e-5,
    out: Optional[torch.Tensor] = None,
    out_dtype: torch.dtype = torch.float16,
    row_len: Optional[torch.Tensor] = None,
    seq_len: int = 0,
    workspace: Optional[torch.Tensor] = None,
):
    """Run one fused GEMM on 2-D row-major operands. Returns ``out`` for
    ``bias``/``gelu``, ``sum_out`` for ``resid`` and ``(sum_out, out)`` for
    ``resid_ln``."""
    if epilogue not in EPILOGUES:
        raise ValueError(f"unknown epilogue {epilogue!r}")
    epi = EPILOGUES[epilogue]
    if a.dim() != 2 or w.dim() != 2 or a.shape[1] != w.shape[1]:
        raise ValueError(f"shape mismatch a{tuple(a.shape)} w{tuple(w.shape)}")
    if a.dtype != torch.float16 or w.dtype != torch.float16:
        raise tk.TKError("linear", -2, "operands must be float16")
    if a.stride(1) != 1 or w.stride(1) != 1:
        raise tk.TKError("linear", -1, "operands need a contiguous last dimension")
    dev = tk.require_cuda(a, w, bias, resid, sum_out, ln_weight, ln_bias, out, row_len)
    M, K = a.shape
    N = w.shape[0]
    bias = bias.float().contiguous()
    if epi in (tk.EPI_BIAS_RESID, tk.EPI_BIAS_RESID_LN):
        if resid is None or resid.dtype != torch.float32:
            raise ValueError("residual epilogues need an fp32 resid")
        if sum_out is None:
            sum_out = torch.empty((M, N), dtype=torch.float32, device=dev)
    if epi != tk.EPI_BIAS_RESID and out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=dev)
    gamma = None if ln_weight is None else ln_weight.float().contiguous()
    beta = None if ln_bias is None else ln_bias.float().contiguous()
    if row_len is not None:
        row_len = row_len.to(torch.int32).contiguous()
    if epi == tk.EPI_BIAS_RESID_LN and N not in (64, 128, 256):
        need = ln_workspace_bytes(M, N)
        if workspace is None:
            workspace = torch.zeros(need, dtype=torch.uint8, device=dev)
        if workspace.dtype != torch.uint8 or workspace.numel() < need or not workspace.is_contiguous():
            raise ValueError(f"workspace must be a contiguous uint8 tensor of >= {need} bytes")
        with torch.cuda.device(dev):
            tk.call(
                "tk_gemm_resid_ln",
                a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0), bias.data_ptr(),
                resid.data_ptr(), resid.stride(0), sum_out.data_ptr(), sum_out.stride(0),
                gamma.data_ptr(), beta.data_ptr(), float(eps),
                out.data_ptr(), tk.dtype_code(out.dtype), out.stride(0),
                tk.ptr(row_len), int(seq_len), M, N, K,
                workspace.data_ptr(), workspace.numel(), tk.stream_handle(dev),
            )
        return sum_out, out
    with torch.cuda.device(dev):
        tk.call(
            "tk_gemm",
            a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0),
            bias.data_ptr(), epi,
            tk.ptr(resid), 0 if resid is None else resid.stride(0),
            tk.ptr(sum_out), 0 if sum_out is None else sum_out.stride(0),
            tk.ptr(gamma), tk.ptr(beta), float(eps),
            tk.ptr(out), tk.dtype_code(out.dtype) if out is not None else tk.TK_F16,
            0 if out is None else out.stride(0),
            tk.ptr(row_len), int(seq_len),
            M, N, K, tk.stream_handle(dev),
        )
    if epi == tk.EPI_BIAS_RESID:
        return sum_out
    if epi == tk.EPI_BIAS_RESID_LN:
        return sum_out, out
    return out
