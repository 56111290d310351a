"""The reference harness's own construction path with the B200 class rebound
in (CPU; skipped where the reference checkout is absent).

The reference swaps its class in by rebinding the harness module's
``UserOptimizedTransformer`` and calling ``main()`` (src/run_case.py:174-201).
``main()`` builds ``UserOptimizedTransformer(config)``, copies the baseline's
weights with a strict ``load_state_dict`` (``copy_model_weights``,
src/torch_transformer_benchmark.py:203-213), moves both models, optionally
compiles the user model (``maybe_compile``, :586-591) and runs the accuracy
loop (``run_accuracy_tests``, :359-424). This test runs exactly those
harness functions with ``GraphedTransformer`` / ``OptimizedTransformer`` in
place, on the CPU of the build container: construction, the strict weight
copy and compilation succeed and copy every weight bit for bit, and the
accuracy loop reaches the B200 forward, which refuses CPU tensors loudly
(there is no CPU path to fall back to). The GPU half of the loop -- the same
seeds, generator and acceptance rule on a B200 -- is
tests/test_model.py::test_c1_five_harness_trials, against the oracle that
tests/test_oracle.py pins to this harness's outputs; the harness itself
does not travel to the GPU box."""

from __future__ import annotations

import importlib.util
import os
import pathlib
import sys

import pytest
import torch

import _tklib as tk
import cuda_graphs
import optimized

HARNESS = pathlib.Path(os.environ.get("TK_REFERENCE_SRC", "/root/reference/src")) / "torch_transformer_benchmark.py"


@pytest.fixture(scope="module")
def bench():
    if not HARNESS.exists():
        pytest.skip("reference harness not present")
    spec = importlib.util.spec_from_file_location("tk_ref_harness", HARNESS)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod  # its dataclasses resolve their module through sys.modules
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("cls", [optimized.OptimizedTransformer, cuda_graphs.GraphedTransformer])
def test_harness_builds_copies_and_reaches_the_b200_forward(bench, cls):
    bench.UserOptimizedTransformer = cls  # the reference's swap, src/run_case.py:182-184
    config = bench.TransformerConfig(batch_size=2, seq_len=16, d_model=64, num_heads=4, ffn_dim=128, num_layers=2,
                                     causal=True)
    config.validate()
    torch.manual_seed(0)
    baseline = bench.BaselineTransformer(config)
    user = bench.UserOptimizedTransformer(config)
    bench.copy_model_weights(baseline, user, strict=True)
    ref_state, got_state = baseline.state_dict(), user.state_dict()
    assert list(ref_state) == list(got_state)
    for key in ref_state:
        assert torch.equal(ref_state[key], got_state[key]), key
    baseline = baseline.to(device="cpu", dtype=torch.float32).eval()
    user = user.to(device="cpu", dtype=torch.float32).eval()
    user = bench.maybe_compile(user, True, "default")  # the harness's --compile-user
    with pytest.raises(tk.TKError, match="CUDA"):
        bench.run_accuracy_tests(baseline, user, config, torch.device("cpu"), torch.float32, trials=1, seed=1234,
                                 padding_ratio=0.0, input_scale=1.0, rtol=0.02, atol=0.002)
