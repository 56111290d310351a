"""tk_layernorm parity (GPU), mirroring the reference's LN tests
(src/test_kernels.py:51-94 and src/test_triton_kernels.py:62-117):
fp16 output within atol 2e-3 / rtol 2e-2, fp32 output within 1e-5, the fp32
residual sum bit-exact, and non-contiguous 3-D inputs."""

from __future__ import annotations

import pytest
import torch

import fused_kernels
from oracle import layer_norm_reference

pytestmark = pytest.mark.gpu


def seeded(*shape, dtype=torch.float32, seed=0, scale=1.0, device="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(device=device, dtype=dtype)


WIDTHS = [32, 33, 64, 100, 128, 512, 768, 1024, 2048, 4096]


@pytest.mark.parametrize("d", WIDTHS)
@pytest.mark.parametrize("residual_dtype", [None, torch.float16, torch.float32])
def test_layernorm_matches_reference(cuda_device, d, residual_dtype):
    rows = 257
    x = seeded(rows, d, seed=d, scale=3.0)
    w = seeded(d, seed=d + 1, scale=0.5) + 1.0
    b = seeded(d, seed=d + 2, scale=0.5)
    if residual_dtype is None:
        y16 = fused_kernels.ln_fwd(x, w, b, 1e-5, torch.float16)
        y32 = fused_kernels.ln_fwd(x, w, b, 1e-5, torch.float32)
        want_sum = x
    else:
        r = seeded(rows, d, dtype=residual_dtype, seed=d + 3)
        s, y16 = fused_kernels.add_ln_fwd(x, r, w, b, 1e-5, torch.float16)
        _, y32 = fused_kernels.add_ln_fwd(x, r, w, b, 1e-5, torch.float32)
        want_sum = x + r.float()
        # the fp32 add is the same IEEE operation: bit-exact
        torch.testing.assert_close(s, want_sum, atol=0.0, rtol=0.0)
    ref = layer_norm_reference(want_sum.cpu(), w.cpu(), b.cpu(), 1e-5, torch.float32)
    torch.testing.assert_close(y16.float().cpu(), ref, atol=2e-3, rtol=2e-2)
    torch.testing.assert_close(y32.cpu(), ref, atol=1e-5, rtol=1e-5)


def test_layernorm_fp16_input(cuda_device):
    x = seeded(64, 512, dtype=torch.float16, seed=5)
    w, b = torch.ones(512, device="cuda"), torch.zeros(512, device="cuda")
    y = fused_kernels.ln_fwd(x, w, b, 1e-5, torch.float32)
    ref = layer_norm_reference(x.float().cpu(), w.cpu(), b.cpu(), 1e-5, torch.float32)
    torch.testing.assert_close(y.cpu(), ref, atol=1e-5, rtol=1e-5)


def test_layernorm_non_contiguous_3d(cuda_device):
    x3 = seeded(4, 16, 128, seed=21).transpose(0, 1)
    w = seeded(128, seed=23) + 1.0
    b = seeded(128, seed=24)
    y = fused_kernels.ln_fwd(x3, w, b, 1e-5, torch.float16)
    assert y.shape == x3.shape
    ref = layer_norm_reference(x3.cpu(), w.cpu(), b.cpu(), 1e-5, torch.float16)
    torch.testing.assert_close(y.cpu().float(), ref.float(), atol=2e-3, rtol=2e-2)


def test_layernorm_leaves_guard_bands_untouched(cuda_device):
    d, rows, pad = 100, 33, 256
    x = seeded(rows, d, seed=9)
    w, b = torch.ones(d, device="cuda"), torch.zeros(d, device="cuda")
    buf = torch.full((rows * d + 2 * pad,), -7.0, dtype=torch.float32, device="cuda")
    out = buf[pad:pad + rows * d].view(rows, d)
    import _tklib as tk

    tk.call("tk_layernorm", x.data_ptr(), 0, d, None, 0, 0, None, 0, w.data_ptr(), b.data_ptr(), 1e-5,
            out.data_ptr(), 0, d, None, 0, rows, d, tk.stream_handle(x.device))
    torch.cuda.synchronize()
    assert torch.all(buf[:pad] == -7.0) and torch.all(buf[-pad:] == -7.0)
    ref = layer_norm_reference(x.cpu(), w.cpu(), b.cpu(), 1e-5, torch.float32)
    torch.testing.assert_close(out.cpu(), ref, atol=1e-5, rtol=1e-5)


# Plain norms with rows * d above the small-launch threshold and 512 < d <= 1024
# (the forward's LN1 / LN2 / final norm) stream each row into shared memory with
# one bulk copy; rows are ragged against the 8-warp blocks, and a strided input
# keeps 16-byte row starts. d = 1020 with fp16 input (2040-byte rows) is not a
# multiple of 16 bytes and takes the per-warp kernel.
@pytest.mark.parametrize("d,x_dtype,out_dtype,pad_cols", [
    (1024, torch.float32, torch.float16, 0),
    (1024, torch.float32, torch.float32, 64),
    (768, torch.float16, torch.float16, 0),
    (1000, torch.float32, torch.float16, 8),
    (1020, torch.float16, torch.float32, 0),
])
def test_layernorm_large_rows(cuda_device, d, x_dtype, out_dtype, pad_cols):
    rows = 6007
    full = seeded(rows, d + pad_cols, dtype=x_dtype, seed=d, scale=3.0)
    x = full[:, :d]
    w = seeded(d, seed=d + 1, scale=0.5) + 1.0
    b = seeded(d, seed=d + 2, scale=0.5)
    y = fused_kernels.ln_fwd(x, w, b, 1e-5, out_dtype)
    ref = layer_norm_reference(x.float().cpu(), w.cpu(), b.cpu(), 1e-5, torch.float32)
    if out_dtype == torch.float32:
        torch.testing.assert_close(y.cpu(), ref, atol=1e-5, rtol=1e-5)
    else:
        torch.testing.assert_close(y.float().cpu(), ref, atol=2e-3, rtol=2e-2)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_layernorm_large_rows_copy_and_padding(cuda_device, out_dtype):
    """The forward's LayerNorm at large row counts (the persistent prefetching
    kernel): the copy of the input rows into the residual buffer is exact,
    and rows past their sequence's prefix length come out as zeros."""
    import _tklib as tk

    S, B, d = 128, 40, 1024
    rows = S * B
    x = seeded(rows, d, seed=41, scale=3.0)
    w = seeded(d, seed=42, scale=0.5) + 1.0
    b = seeded(d, seed=43, scale=0.5)
    lengths = ((torch.arange(B, dtype=torch.int32) * 37) % (S + 1)).cuda()
    copy = torch.full((rows, d), 5.0, device="cuda")
    out = torch.empty(rows, d, dtype=out_dtype, device="cuda")
    tk.call("tk_layernorm", x.data_ptr(), tk.TK_F32, d, None, 0, 0, copy.data_ptr(), d, w.data_ptr(), b.data_ptr(),
            1e-5, out.data_ptr(), tk.dtype_code(out_dtype), d, lengths.data_ptr(), S, rows, d,
            tk.stream_handle(cuda_device))
    torch.cuda.synchronize()
    torch.testing.assert_close(copy, x, atol=0, rtol=0)
    pad = ((torch.arange(rows) % S) >= lengths.cpu().repeat_interleave(S))
    got = out.float().cpu()
    assert torch.all(got[pad] == 0)
    ref = layer_norm_reference(x.cpu(), w.cpu(), b.cpu(), 1e-5, torch.float32)
    tol = dict(atol=2e-3, rtol=2e-2) if out_dtype == torch.float16 else dict(atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(got[~pad], ref[~pad], **tol)
