"""fp32 CPU restatement of the harness model, inputs and acceptance rule.

TEST INFRASTRUCTURE ONLY (see the package docstring): the product never
imports this module.

Every function cites the line range of the organisers' harness
``src/torch_transformer_benchmark.py`` (danielfodgaard/transformer-kernel) or
of the reference's test files whose behaviour it restates. The model is
written as plain functions over a ``state_dict`` (the harness's parameter
names), so the oracle owns no ``nn.Module`` forward; ``nn.Linear`` and
``nn.LayerNorm`` are only instantiated to consume the global RNG exactly as
the harness's constructors do, which reproduces its default initialisation
bit for bit.

Parity is pinned: ``tests/test_oracle.py`` checks ``init_params``,
``generate_random_case`` and ``stack_forward`` against fixtures produced by
the unmodified reference harness (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import math
from collections import OrderedDict
from dataclasses import dataclass
from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

Params = Dict[str, torch.Tensor]


@dataclass(frozen=True)
class StackConfig:
    """Shape of one layer stack; same fields as the harness's
    ``TransformerConfig`` (``src/torch_transformer_benchmark.py:29-56``)."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads

    @property
    def tokens(self) -> int:
        return self.batch_size * self.seq_len


# --------------------------------------------------------------------------- #
# Weights
# --------------------------------------------------------------------------- #


def init_params(cfg: StackConfig, seed: int = 0) -> Params:
    """Default-initialised weights under ``torch.manual_seed(seed)``.

    RNG consumption follows the harness constructors: per block
    ``norm1, q_proj, k_proj, v_proj, out_proj, norm2, ffn_in, ffn_out``
    (``:125-132`` and ``:72-75``), blocks in order, then ``final_norm``
    (``:150-160``). Keys are the harness's ``state_dict`` keys.
    """
    torch.manual_seed(seed)
    d, f = cfg.d_model, cfg.ffn_dim
    params: Params = OrderedDict()

    def put(prefix: str, module: nn.Module) -> None:
        for name, tensor in module.state_dict().items():
            params[f"{prefix}.{name}"] = tensor.detach().clone()

    for i in range(cfg.num_layers):
        p = f"layers.{i}"
        put(f"{p}.norm1", nn.LayerNorm(d))
        for proj in ("q_proj", "k_proj", "v_proj", "out_proj"):
            put(f"{p}.attention.{proj}", nn.Linear(d, d, bias=True))
        put(f"{p}.norm2", nn.LayerNorm(d))
        put(f"{p}.ffn_in", nn.Linear(d, f))
        put(f"{p}.ffn_out", nn.Linear(f, d))
    put("final_norm", nn.LayerNorm(d))
    return params


# --------------------------------------------------------------------------- #
# Inputs
# --------------------------------------------------------------------------- #


def generate_random_case(
    cfg: StackConfig,
    seed: int,
    padding_ratio: float = 0.0,
    input_scale: float = 1.0,
    device: str = "cpu",
    dtype: torch.dtype = torch.float32,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Seeded ``(x, valid_token_mask)`` (``:234-272``).

    Draw order on one generator: ``randn(B,S,d)`` first, then (only with
    padding) ``randint`` lengths in ``[round(S*(1-p)) clamped >= 1, S]``; the
    mask is a per-row prefix and padded rows of ``x`` are zeroed.
    """
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    shape = (cfg.batch_size, cfg.seq_len, cfg.d_model)
    x = torch.randn(*shape, generator=gen, device=device, dtype=dtype) * input_scale
    if padding_ratio <= 0:
        mask = torch.ones(cfg.batch_size, cfg.seq_len, device=device, dtype=torch.bool)
        return x, mask
    shortest = max(1, int(round(cfg.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(
        low=shortest, high=cfg.seq_len + 1, size=(cfg.batch_size,),
        generator=gen, device=device,
    )
    mask = torch.arange(cfg.seq_len, device=device)[None, :] < lengths[:, None]
    return x.masked_fill(~mask[..., None], 0), mask


# --------------------------------------------------------------------------- #
# Model
# --------------------------------------------------------------------------- #


def _heads(t: torch.Tensor, n_heads: int) -> torch.Tensor:
    """``[B,S,d] -> [B,H,S,hd]`` contiguous (``:77-83``)."""
    b, s, d = t.shape
    return t.view(b, s, n_heads, d // n_heads).transpose(1, 2).contiguous()


def _self_attention(
    params: Params, prefix: str, h: torch.Tensor, n_heads: int,
    mask: Optional[torch.Tensor], causal: bool,
) -> torch.Tensor:
    """Explicit multi-head attention in the harness's op order (``:85-122``):
    separate Q/K/V projections, fp32-matmul scores multiplied by
    ``hd**-0.5`` after the matmul, ``-inf`` for the strict upper triangle and
    for invalid keys, softmax in fp32, ``probs @ v``, merge heads, output
    projection, zero the rows of invalid queries."""
    b, s, d = h.shape
    w = lambda name: params[f"{prefix}.{name}"]  # noqa: E731
    q = _heads(F.linear(h, w("q_proj.weight"), w("q_proj.bias")), n_heads)
    k = _heads(F.linear(h, w("k_proj.weight"), w("k_proj.bias")), n_heads)
    v = _heads(F.linear(h, w("v_proj.weight"), w("v_proj.bias")), n_heads)
    scale = (d // n_heads) ** -0.5
    scores = torch.matmul(q, k.transpose(-2, -1)) * scale
    if causal:
        upper = torch.ones((s, s), dtype=torch.bool, device=h.device).triu(diagonal=1)
        scores = scores.masked_fill(upper, float("-inf"))
    if mask is not None:
        scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores.float(), dim=-1).to(dtype=h.dtype)
    ctx = torch.matmul(probs, v).transpose(1, 2).contiguous().view(b, s, d)
    out = F.linear(ctx, w("out_proj.weight"), w("out_proj.bias"))
    if mask is not None:
        out = out.masked_fill(~mask[..., None], 0)
    return out


def _block(
    params: Params, i: int, cfg: StackConfig, x: torch.Tensor,
    mask: Optional[torch.Tensor],
) -> torch.Tensor:
    """Pre-LN block (``:134-145``): ``x += Attn(LN1 x)``;
    ``x += W2 gelu_erf(W1 LN2 x + b1) + b2``; zero padded rows."""
    p = f"layers.{i}"
    d = cfg.d_model

    def ln(name: str, t: torch.Tensor) -> torch.Tensor:
        return F.layer_norm(t, (d,), params[f"{p}.{name}.weight"], params[f"{p}.{name}.bias"], 1e-5)

    x = x + _self_attention(params, f"{p}.attention", ln("norm1", x), cfg.num_heads, mask, cfg.causal)
    hidden = F.gelu(
        F.linear(ln("norm2", x), params[f"{p}.ffn_in.weight"], params[f"{p}.ffn_in.bias"]),
        approximate="none",
    )
    x = x + F.linear(hidden, params[f"{p}.ffn_out.weight"], params[f"{p}.ffn_out.bias"])
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
    return x


@torch.inference_mode()
def stack_forward(
    params: Params, cfg: StackConfig, x: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """``BaselineTransformer.forward`` (``:162-172``): all blocks, then
    ``final_norm``, then zero padded rows. Computes in ``x``'s dtype (fp32
    for every configuration this build grades)."""
    for i in range(cfg.num_layers):
        x = _block(params, i, cfg, x, valid_token_mask)
    x = F.layer_norm(x, (cfg.d_model,), params["final_norm.weight"], params["final_norm.bias"], 1e-5)
    if valid_token_mask is not None:
        x = x.masked_fill(~valid_token_mask[..., None], 0)
    return x


@torch.inference_mode()
def chunked_forward(
    params: Params, cfg: StackConfig, x: torch.Tensor,
    valid_token_mask: Optional[torch.Tensor] = None, chunk: int = 1,
) -> torch.Tensor:
    """Batch-chunked ``stack_forward``. Batch rows never interact, so this
    is exact; it bounds the ``[B,H,S,S]`` score tensor the way the
    reference's out-of-core runner does (``src/run_case14.py:153-158``)."""
    outs = []
    for start in range(0, x.shape[0], chunk):
        m = None if valid_token_mask is None else valid_token_mask[start:start + chunk]
        outs.append(stack_forward(params, cfg, x[start:start + chunk], m))
    return torch.cat(outs, dim=0)


def _attention_rows(
    params: Params, prefix: str, h: torch.Tensor, rows: torch.Tensor, n_heads: int,
    mask: Optional[torch.Tensor], causal: bool, q_chunk: int,
) -> torch.Tensor:
    """``_self_attention`` for the query positions ``rows`` only, with the
    scores of ``q_chunk`` queries at a time (never the ``[S, S]`` matrix):
    the exact, query-chunked fp32 attention that the reference's long-sequence
    runner uses as its stand-in for the baseline (``src/run_case14.py:57-62``,
    validated against the baseline at ``:165-221``). Same op order as
    ``:85-122``; returns ``[B, len(rows), d]``."""
    b, s, d = h.shape
    w = lambda name: params[f"{prefix}.{name}"]  # noqa: E731
    k = _heads(F.linear(h, w("k_proj.weight"), w("k_proj.bias")), n_heads)
    v = _heads(F.linear(h, w("v_proj.weight"), w("v_proj.bias")), n_heads)
    q = _heads(F.linear(h[:, rows], w("q_proj.weight"), w("q_proj.bias")), n_heads)
    scale = (d // n_heads) ** -0.5
    key_pos = torch.arange(s, device=h.device)
    ctx = []
    for start in range(0, rows.numel(), q_chunk):
        pos = rows[start:start + q_chunk]
        scores = torch.matmul(q[:, :, start:start + q_chunk], k.transpose(-2, -1)) * scale
        if causal:
            scores = scores.masked_fill(key_pos[None, :] > pos[:, None], float("-inf"))
        if mask is not None:
            scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
        probs = torch.softmax(scores.float(), dim=-1).to(dtype=h.dtype)
        ctx.append(torch.matmul(probs, v).transpose(1, 2).reshape(b, pos.numel(), d))
    out = F.linear(torch.cat(ctx, dim=1), w("out_proj.weight"), w("out_proj.bias"))
    if mask is not None:
        out = out.masked_fill(~mask[:, rows][..., None], 0)
    return out


def _block_rows(
    params: Params, i: int, cfg: StackConfig, x: torch.Tensor,
    mask: Optional[torch.Tensor], rows: torch.Tensor, q_chunk: int,
) -> torch.Tensor:
    """``_block`` evaluated at the positions ``rows`` (every position feeds
    the keys and values): returns ``[B, len(rows), d]``."""
    p = f"layers.{i}"
    d = cfg.d_model

    def ln(name: str, t: torch.Tensor) -> torch.Tensor:
        return F.layer_norm(t, (d,), params[f"{p}.{name}.weight"], params[f"{p}.{name}.bias"], 1e-5)

    h = ln("norm1", x)
    y = x[:, rows] + _attention_rows(params, f"{p}.attention", h, rows, cfg.num_heads, mask, cfg.causal, q_chunk)
    hidden = F.gelu(
        F.linear(ln("norm2", y), params[f"{p}.ffn_in.weight"], params[f"{p}.ffn_in.bias"]),
        approximate="none",
    )
    y = y + F.linear(hidden, params[f"{p}.ffn_out.weight"], params[f"{p}.ffn_out.bias"])
    if mask is not None:
        y = y.masked_fill(~mask[:, rows][..., None], 0)
    return y


@torch.inference_mode()
def stack_forward_rows(
    params: Params, cfg: StackConfig, x: torch.Tensor, rows: Optional[torch.Tensor] = None,
    valid_token_mask: Optional[torch.Tensor] = None, q_chunk: int = 256,
) -> torch.Tensor:
    """Rows ``rows`` (sequence positions, default all) of ``stack_forward``,
    computed with query-chunked exact attention so long sequences never form
    an ``[S, S]`` score matrix -- the reference's proxy for sequences the
    baseline cannot hold (``src/run_case14.py:57-62,165-221``). Layers before
    the last run at every position; the last one only at ``rows``, which is
    exact because a layer's output row depends on other rows only through
    the keys and values. Returns ``[B, len(rows), d]``."""
    s = x.shape[1]
    every = torch.arange(s)
    rows = every if rows is None else rows.to(torch.long)
    for i in range(cfg.num_layers):
        last = i == cfg.num_layers - 1
        x = _block_rows(params, i, cfg, x, valid_token_mask, rows if last else every, q_chunk)
    x = F.layer_norm(x, (cfg.d_model,), params["final_norm.weight"], params["final_norm.bias"], 1e-5)
    if valid_token_mask is not None:
        x = x.masked_fill(~valid_token_mask[:, rows][..., None], 0)
    return x


# --------------------------------------------------------------------------- #
# Kernel-level references
# --------------------------------------------------------------------------- #


def layer_norm_reference(
    x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float,
    out_dtype: torch.dtype,
) -> torch.Tensor:
    """fp32 LayerNorm then the cast (``src/test_kernels.py:30-41``)."""
    y = F.layer_norm(x.float(), (x.shape[-1],), weight.float(), bias.float(), eps)
    return y.to(out_dtype)


def attention_reference(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
    causal: bool, kv_len: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Baseline-order attention on ``[B,H,S,hd]`` inputs returning
    ``[B,S,H*hd]`` fp32 (``src/test_triton_kernels.py:125-139``): fp32
    scores, post-scale, ``-inf`` strict upper triangle, fp32 softmax, PV in
    fp32. ``kv_len[b]`` optionally masks keys ``>= kv_len[b]`` (the harness's
    prefix key-padding mask, ``:101-104``)."""
    qf, kf, vf = q.float(), k.float(), v.float()
    s = q.shape[-2]
    scores = torch.matmul(qf, kf.transpose(-2, -1)) * scale
    if causal:
        upper = torch.ones((s, s), dtype=torch.bool, device=q.device).triu(diagonal=1)
        scores = scores.masked_fill(upper, float("-inf"))
    if kv_len is not None:
        invalid = torch.arange(s, device=q.device)[None, :] >= kv_len.to(q.device)[:, None]
        scores = scores.masked_fill(invalid[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    ctx = torch.matmul(probs, vf)
    b, h, _, hd = ctx.shape
    return ctx.transpose(1, 2).reshape(b, s, h * hd)


# --------------------------------------------------------------------------- #
# Acceptance rule
# --------------------------------------------------------------------------- #


@dataclass
class AccuracyResult:
    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float
    worst_index: Tuple[int, ...]


def compare_outputs(
    reference: torch.Tensor, candidate: torch.Tensor, rtol: float = 0.02,
    atol: float = 0.002,
) -> AccuracyResult:
    """The harness's element rule (``:289-356``; defaults ``:618-619``):
    every element must be finite on both sides and satisfy
    ``|u-r| <= atol OR |u-r| <= rtol*|r|`` -- an OR of the two bounds, not
    ``isclose``'s sum."""
    if reference.shape != candidate.shape:
        raise AssertionError(f"shape mismatch: {tuple(reference.shape)} vs {tuple(candidate.shape)}")
    ref = reference.detach().float().cpu()
    cand = candidate.detach().float().cpu()
    err = (cand - ref).abs()
    ok = torch.isfinite(ref) & torch.isfinite(cand) & ((err <= atol) | (err <= rtol * ref.abs()))
    failed = int((~ok).sum())
    flat = int(err.reshape(-1).nan_to_num(nan=math.inf).argmax())
    worst = []
    for size in reversed(ref.shape):
        worst.append(flat % size)
        flat //= size
    rel = err / ref.abs().clamp_min(1e-12)
    return AccuracyResult(
        passed=failed == 0,
        total_elements=ref.numel(),
        failed_elements=failed,
        max_abs_error=float(err.max()) if err.numel() else 0.0,
        max_relative_error=float(rel.max()) if rel.numel() else 0.0,
        mean_abs_error=float(err.mean()) if err.numel() else 0.0,
        worst_index=tuple(reversed(worst)),
    )
