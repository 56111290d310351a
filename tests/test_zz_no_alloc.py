"""The allocation-free GEMM + residual + LayerNorm entry point (GPU).

Some callers cannot allocate device memory -- a plugin whose host framework
owns every device allocation, a serving loop that may not call the
allocator once it runs -- so they cannot hand tk_gemm_resid_ln its
workspace. tk_gemm_resid_ln_static takes no workspace and uses a fixed 8 MiB
array inside the library instead. This file checks, through the C ABI, that
it gives the same sum and LayerNorm output as tk_gemm_resid_ln with a
workspace, on two calls in a row (the shared array keeps the previous
call's contents, which each call must clear), and that it refuses a size
beyond its array before launching anything.

Collected last on purpose (the file name): a failure here leaves every
other test already run when pytest stops at the first failure.
"""

from __future__ import annotations

import pytest
import torch

import _tklib as tk
import linear as tk_linear

pytestmark = pytest.mark.gpu


def _case(M, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).half().cuda()
    w = (torch.randn(N, K, generator=g) * K ** -0.5).half().cuda()
    b = (torch.randn(N, generator=g) * 0.1).cuda()
    r = torch.randn(M, N, generator=g).cuda()
    gamma = (torch.randn(N, generator=g) * 0.5 + 1.0).cuda()
    beta = (torch.randn(N, generator=g) * 0.5).cuda()
    return a, w, b, r, gamma, beta


def _args(a, w, b, resid, s, gamma, beta, h):
    M, K = a.shape
    N = w.shape[0]
    return (a.data_ptr(), K, w.data_ptr(), K, b.data_ptr(), resid.data_ptr(), N, s.data_ptr(), N,
            gamma.data_ptr(), beta.data_ptr(), 1e-5, h.data_ptr(), tk.dtype_code(h.dtype), N, None, 0, M, N, K)


@pytest.mark.parametrize("M,N,K,out_dtype", [(65536, 1024, 1024, torch.float16), (3001, 512, 2048, torch.float32)])
def test_static_scratch_matches_workspace_entry_point(cuda_device, M, N, K, out_dtype):
    stream = tk.stream_handle(cuda_device)
    ws = torch.zeros(tk_linear.ln_workspace_bytes(M, N), dtype=torch.uint8, device=cuda_device)
    for call, seed in enumerate((11, 12)):  # two calls in a row, different data
        a, w, b, r, gamma, beta = _case(M, N, K, seed + 100 * N)
        s_ref, s_new = r.clone(), r.clone()  # the residual stream, updated in place
        h_ref = torch.empty(M, N, dtype=out_dtype, device=cuda_device)
        h_new = torch.full((M, N), 7.0, dtype=out_dtype, device=cuda_device)
        tk.call("tk_gemm_resid_ln", *_args(a, w, b, s_ref, s_ref, gamma, beta, h_ref), ws.data_ptr(), ws.numel(),
                stream)
        tk.call("tk_gemm_resid_ln_static", *_args(a, w, b, s_new, s_new, gamma, beta, h_new), stream)
        torch.cuda.synchronize()
        torch.testing.assert_close(s_new, s_ref, atol=1e-4, rtol=1e-4, msg=f"call {call}: sum")
        tol = dict(atol=2e-3, rtol=2e-2) if out_dtype == torch.float16 else dict(atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(h_new.float(), h_ref.float(), **tol, msg=f"call {call}: LayerNorm output")


def test_static_scratch_refuses_rows_beyond_its_array(cuda_device):
    M, N, K = 200000, 1024, 64  # needs 14.4 MB of scratch, the array holds 8 MiB
    x = torch.zeros(16, device=cuda_device)
    p = x.data_ptr()
    rc = tk.lib().tk_gemm_resid_ln_static(p, K, p, K, p, p, N, p, N, p, p, 1e-5, p, tk.TK_F16, N, None, 0, M, N, K,
                                          tk.stream_handle(cuda_device))
    assert rc == -2
    assert b"scratch" in tk.lib().tk_last_error()
