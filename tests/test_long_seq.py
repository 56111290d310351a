"""Long-sequence parity (GPU): the out-of-core-scale configuration's
sequence length (S = 100,000, d 1024, 16 heads, ffn 4096, one causal layer)
run in-core on one GPU, one or two samples at a time, and checked at spot
rows against the exact query-chunked fp32 oracle -- the reference's own
stand-in for a baseline that cannot hold the [S, S] scores
(src/run_case14.py:57-62,165-221) -- under the harness rule."""

from __future__ import annotations

import pytest
import torch

import optimized
from oracle import StackConfig, compare_outputs, generate_random_case, init_params, stack_forward_rows

pytestmark = pytest.mark.gpu

RTOL, ATOL = 0.02, 0.002


def spot_rows(S: int, extra: int = 16, seed: int = 7) -> torch.Tensor:
    """Tile edges, both ends of the sequence, and seeded random positions."""
    fixed = [0, 1, 127, 128, 129, 255, 4095, 4096, S // 2, S - 129, S - 128, S - 2, S - 1]
    g = torch.Generator().manual_seed(seed)
    rnd = torch.randint(0, S, (extra,), generator=g).tolist()
    return torch.tensor(sorted({r for r in fixed + rnd if 0 <= r < S}))


def run_spot_check(cfg: StackConfig, seed: int, padding_ratio: float = 0.0):
    params = init_params(cfg, seed=0)
    model = optimized.OptimizedTransformer(cfg)
    model.load_state_dict(params, strict=True)
    model = model.cuda().eval()
    x, mask = generate_random_case(cfg, seed, padding_ratio)
    with torch.inference_mode():
        out = model(x.cuda(), mask.cuda()).cpu()
    rows = spot_rows(cfg.seq_len)
    ref = stack_forward_rows(params, cfg, x, rows, None if padding_ratio == 0 else mask, q_chunk=8)
    r = compare_outputs(ref, out[:, rows], RTOL, ATOL)
    assert r.passed, str(r)
    return r


def test_c5_sequence_length_one_sample(cuda_device):
    run_spot_check(StackConfig(1, 100000, 1024, 16, 4096, 1, True), seed=1234)


def test_long_sequence_padded_two_samples(cuda_device):
    # prefix key-padding masks at long S (the kv-bound path of the attention)
    run_spot_check(StackConfig(2, 30000, 1024, 16, 4096, 1, True), seed=1235, padding_ratio=0.3)
