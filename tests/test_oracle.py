"""Pin the CPU oracle against the unmodified reference harness.

The fixtures in ``tests/golden/golden.pt`` were produced by importing the
reference's ``src/torch_transformer_benchmark.py`` (see
``tests/golden/make_golden.py``). Weights and inputs must match exactly;
outputs to 1e-5 (the oracle runs the same fp32 CPU ops in the same order,
the slack only absorbs BLAS thread-count differences).
"""

from __future__ import annotations

import pytest
import torch

from oracle import StackConfig, compare_outputs, generate_random_case, init_params, stack_forward, stack_forward_rows

SMALL = ["tiny_causal", "tiny_bidir", "tiny_padded", "ragged_s"]
LARGE = ["c1_reference_case1", "c2_small_batch", "c3_slice_b2_l1", "c4_slice_s1024_l1"]


def _case(golden, name):
    entry = golden[name]
    cfg = StackConfig(**entry["config"])
    params = init_params(cfg, seed=0)
    x, mask = generate_random_case(cfg, entry["input_seed"], entry["padding_ratio"])
    return entry, cfg, params, x, mask


@pytest.mark.parametrize("name", SMALL + LARGE)
def test_weights_and_inputs_match_harness(golden, name):
    entry, cfg, params, x, mask = _case(golden, name)
    assert list(params.keys()) == entry["weight_keys"]
    for key, (s, a) in entry["weight_checksums"].items():
        t = params[key].double()
        assert float(t.sum()) == s and float(t.abs().sum()) == a, key
    assert (float(x.double().sum()), float(x.double().abs().sum())) == tuple(entry["x_checksum"])
    assert torch.equal(mask, entry["mask"])


@pytest.mark.parametrize("name", SMALL)
def test_forward_matches_harness_small(golden, name):
    entry, cfg, params, x, mask = _case(golden, name)
    out = stack_forward(params, cfg, x, mask)
    torch.testing.assert_close(out, entry["out"], atol=1e-5, rtol=0)


@pytest.mark.parametrize("name", LARGE)
def test_forward_matches_harness_large(golden, name):
    entry, cfg, params, x, mask = _case(golden, name)
    out = stack_forward(params, cfg, x, mask)
    torch.testing.assert_close(out.double().sum(-1).float(), entry["out_row_sums"], atol=2e-4, rtol=0)
    got = torch.stack([out[i, j] for i, j in entry["out_rows_index"]])
    torch.testing.assert_close(got, entry["out_rows"], atol=1e-5, rtol=0)


def test_acceptance_rule_is_or_not_isclose():
    ref = torch.tensor([1.0, 0.0, 10.0, float("nan")])
    # 0.15 abs error on 10.0 passes only through rtol (0.02*10 = 0.2)
    cand = torch.tensor([1.0019, 0.0021, 10.15, float("nan")])
    r = compare_outputs(ref[:3], cand[:3])
    assert r.failed_elements == 1  # 0.0021 > atol and > rtol*0
    assert not compare_outputs(ref, ref.clone()).passed  # non-finite fails


def test_acceptance_rule_catches_a_planted_error(golden):
    entry, cfg, params, x, mask = _case(golden, "tiny_causal")
    out = stack_forward(params, cfg, x, mask)
    bad = out.clone()
    bad[1, 3, 7] += 0.01 + 0.05 * bad[1, 3, 7].abs()
    r = compare_outputs(entry["out"], bad)
    assert not r.passed and r.failed_elements == 1 and r.worst_index == (1, 3, 7)


@pytest.mark.parametrize("causal", [True, False])
def test_query_chunked_rows_match_stack_forward(causal):
    """The query-chunked row-subset oracle (the long-sequence proxy) equals
    the full-matrix oracle, masks included, for every row subset and chunk."""
    cfg = StackConfig(2, 300, 64, 4, 128, 2, causal)
    params = init_params(cfg, seed=0)
    x, mask = generate_random_case(cfg, seed=5)
    mask[1, 200:] = False
    full = stack_forward(params, cfg, x, mask)
    rows = torch.tensor([0, 1, 63, 64, 150, 199, 200, 299])
    got = stack_forward_rows(params, cfg, x, rows, mask, q_chunk=3)
    torch.testing.assert_close(got, full[:, rows], atol=1e-6, rtol=1e-6)
    torch.testing.assert_close(stack_forward_rows(params, cfg, x, None, mask, q_chunk=64), full,
                               atol=1e-6, rtol=1e-6)
