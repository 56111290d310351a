"""Failure detection without a GPU fault: a kernel waits on an mbarrier that
nothing arrives on; its bounded wait must give up, record the failure in
the device error word, and leave the context usable."""

from __future__ import annotations

import pytest
import torch

import _tklib as tk
import fused_kernels

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives(cuda_device):
    old = tk.set_wait_limit_ns(2_000_000)  # 2 ms
    try:
        tk.call("tk_selftest_wait_timeout", tk.stream_handle(cuda_device))
        with pytest.raises(tk.TKError) as err:
            tk.check_device_errors(cuda_device)
        assert err.value.status == -4 and "timed out" in str(err.value)
        # the error word is cleared once read
        tk.check_device_errors(cuda_device)
    finally:
        tk.set_wait_limit_ns(old)
    x = torch.randn(16, 128, device="cuda")
    y = fused_kernels.ln_fwd(x, torch.ones(128, device="cuda"), torch.zeros(128, device="cuda"), 1e-5)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
