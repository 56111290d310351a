"""tk_gemm parity (GPU): every epilogue against an fp32 CPU reference on the
same fp16-rounded operands. The GEMM accumulates exact fp16 products in
fp32, so fp32 outputs agree to ~1e-4 relative and fp16 outputs to fp16
rounding (atol 2e-3, rtol 2e-2, the reference's fp16 budget)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

import linear as tk_linear

pytestmark = pytest.mark.gpu


def seeded(*shape, seed=0, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g) * scale


def operands(M, N, K, seed):
    a = seeded(M, K, seed=seed).half()
    w = (seeded(N, K, seed=seed + 1) * K ** -0.5).half()
    b = seeded(N, seed=seed + 2) * 0.1
    return a, w, b


def ref_linear(a, w, b):
    return a.float() @ w.float().t() + b


# (M, N, K): model GEMM shapes of the configs (QKV, O, FFN-in, FFN-out), plus ragged M
SHAPES = [
    (8192, 384, 128), (8192, 128, 128),           # C1
    (512, 1536, 512), (512, 512, 512), (512, 2048, 512), (512, 512, 2048),  # C2
    (2048, 3072, 1024), (2048, 1024, 4096), (2048, 4096, 1024),            # C3/C4 (M cut)
    (300, 256, 64), (129, 96, 200), (1, 64, 8),                            # ragged
]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_bias(cuda_device, M, N, K):
    a, w, b = operands(M, N, K, seed=M + N + K)
    out = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "bias")
    torch.testing.assert_close(out.float().cpu(), ref_linear(a, w, b), atol=2e-3, rtol=2e-2)


@pytest.mark.parametrize("M,N,K", [(512, 2048, 512), (2048, 4096, 1024), (129, 96, 200)])
def test_gemm_bias_gelu(cuda_device, M, N, K):
    a, w, b = operands(M, N, K, seed=7)
    out = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "gelu")
    want = F.gelu(ref_linear(a, w, b), approximate="none")
    # tight: fp16 output rounding (2^-11 relative) plus the A&S 7.1.26 erf
    # error (<= 1.5e-7); a looser erf would show here
    torch.testing.assert_close(out.float().cpu(), want, atol=2e-4, rtol=1e-3)


def test_gemm_gelu_extreme_inputs(cuda_device):
    """GELU tails: large |x| saturates to x or 0, tiny |x| stays ~x/2."""
    M, N, K = 128, 64, 16
    a = torch.zeros(M, K, dtype=torch.float16)
    w = torch.zeros(N, K, dtype=torch.float16)
    b = torch.cat([torch.linspace(-12, 12, N - 8), torch.tensor([1e-4, -1e-4, 3e-3, -3e-3, 0.5, -0.5, 7.0, -7.0])])
    out = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "gelu").float().cpu()
    want = F.gelu(b, approximate="none").expand(M, N)
    torch.testing.assert_close(out, want, atol=2e-6, rtol=1e-3)


@pytest.mark.parametrize("M,N,K", [(512, 512, 2048), (2048, 1024, 4096), (300, 256, 64), (129, 96, 200)])
def test_gemm_bias_resid(cuda_device, M, N, K):
    a, w, b = operands(M, N, K, seed=11)
    r = seeded(M, N, seed=12)
    s = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid", resid=r.cuda())
    torch.testing.assert_close(s.cpu(), r + ref_linear(a, w, b), atol=1e-4, rtol=1e-4)


def test_gemm_bias_resid_in_place(cuda_device):
    a, w, b = operands(1024, 512, 512, seed=13)
    r = seeded(1024, 512, seed=14)
    buf = r.cuda()
    s = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid", resid=buf, sum_out=buf)
    assert s.data_ptr() == buf.data_ptr()
    torch.testing.assert_close(buf.cpu(), r + ref_linear(a, w, b), atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("M,N,K", [(8192, 128, 128), (1000, 64, 256), (512, 256, 1024)])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_gemm_bias_resid_layernorm(cuda_device, M, N, K, out_dtype):
    a, w, b = operands(M, N, K, seed=17)
    r = seeded(M, N, seed=18)
    g = seeded(N, seed=19, scale=0.5) + 1.0
    beta = seeded(N, seed=20, scale=0.5)
    s, h = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid_ln", resid=r.cuda(), ln_weight=g.cuda(),
                            ln_bias=beta.cuda(), eps=1e-5, out_dtype=out_dtype)
    want_s = r + ref_linear(a, w, b)
    torch.testing.assert_close(s.cpu(), want_s, atol=1e-4, rtol=1e-4)
    want_h = F.layer_norm(want_s, (N,), g, beta, 1e-5)
    tol = dict(atol=2e-3, rtol=2e-2) if out_dtype == torch.float16 else dict(atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(h.float().cpu(), want_h, **tol)


def test_gemm_row_len_zeroes_padded_rows(cuda_device):
    S, B, N, K = 64, 3, 128, 128
    a, w, b = operands(B * S, N, K, seed=23)
    r = seeded(B * S, N, seed=24)
    lengths = torch.tensor([64, 10, 1], dtype=torch.int32)
    s, h = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid_ln", resid=r.cuda(),
                            ln_weight=torch.ones(N).cuda(), ln_bias=torch.zeros(N).cuda(),
                            out_dtype=torch.float32, row_len=lengths.cuda(), seq_len=S)
    pos = torch.arange(B * S) % S
    pad = pos >= lengths.repeat_interleave(S)
    assert torch.all(s.cpu()[pad] == 0) and torch.all(h.cpu()[pad] == 0)
    want_s = r + ref_linear(a, w, b)
    torch.testing.assert_close(s.cpu()[~pad], want_s[~pad], atol=1e-4, rtol=1e-4)


def test_gemm_output_guard_bands(cuda_device):
    M, N, K, pad = 200, 96, 64, 4096
    a, w, b = operands(M, N, K, seed=29)
    buf = torch.full((M * N + 2 * pad,), 123.0, dtype=torch.float16, device="cuda")
    out = buf[pad:pad + M * N].view(M, N)
    tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "bias", out=out)
    torch.cuda.synchronize()
    assert torch.all(buf[:pad] == 123.0) and torch.all(buf[-pad:] == 123.0)
    torch.testing.assert_close(out.float().cpu(), ref_linear(a, w, b), atol=2e-3, rtol=2e-2)


# Shapes with N % 256 == 0 and >= 148 tiles of 256 x 256 take the CTA-pair
# (tcgen05 cta_group::2) kernel; the M tails leave the odd CTA of the last
# pair partly (9000) or entirely (8320) out of range.
PAIR_SHAPES = [(8192, 3072, 1024), (9000, 2048, 512), (8320, 4096, 256)]


@pytest.mark.parametrize("M,N,K", PAIR_SHAPES)
def test_gemm_pair_bias(cuda_device, M, N, K):
    a, w, b = operands(M, N, K, seed=31)
    out = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "bias")
    torch.testing.assert_close(out.float().cpu(), ref_linear(a, w, b), atol=2e-3, rtol=2e-2)


@pytest.mark.parametrize("M,N,K", PAIR_SHAPES[1:])
def test_gemm_pair_gelu(cuda_device, M, N, K):
    a, w, b = operands(M, N, K, seed=37)
    out = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "gelu")
    want = F.gelu(ref_linear(a, w, b), approximate="none")
    torch.testing.assert_close(out.float().cpu(), want, atol=2e-4, rtol=1e-3)


@pytest.mark.parametrize("M,N,K", [(16384, 1024, 1024), (9000, 2048, 512)])
def test_gemm_pair_resid_in_place(cuda_device, M, N, K):
    a, w, b = operands(M, N, K, seed=41)
    r = seeded(M, N, seed=42)
    buf = r.cuda()
    tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid", resid=buf, sum_out=buf)
    torch.testing.assert_close(buf.cpu(), r + ref_linear(a, w, b), atol=1e-4, rtol=1e-4)


def test_gemm_pair_resid_in_place_strided_guard_bands(cuda_device):
    # The residual stream as a strided window of a guarded fp32 buffer: the
    # TMA reduce-adds touch exactly the M x N window (the M tail is clipped,
    # the columns past N and the guard bands keep their sentinel).
    M, N, K, ld, pad = 9000, 1024, 512, 1024 + 32, 4096
    a, w, b = operands(M, N, K, seed=61)
    r = seeded(M, N, seed=62)
    buf = torch.full((M * ld + 2 * pad,), -5.0, dtype=torch.float32, device="cuda")
    win = buf[pad:pad + M * ld].view(M, ld)[:, :N]
    win.copy_(r.cuda())
    tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid", resid=win, sum_out=win)
    torch.cuda.synchronize()
    host = buf.cpu()
    assert torch.all(host[:pad] == -5.0) and torch.all(host[-pad:] == -5.0)
    assert torch.all(host[pad:pad + M * ld].view(M, ld)[:, N:] == -5.0)
    torch.testing.assert_close(win.cpu(), r + ref_linear(a, w, b), atol=1e-4, rtol=1e-4)


def test_gemm_pair_k_tail(cuda_device):
    # K = 320: the last 128-wide k stage of the pair kernel is half zero-filled
    M, N, K = 8192, 2048, 320
    a, w, b = operands(M, N, K, seed=43)
    out = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "bias")
    torch.testing.assert_close(out.float().cpu(), ref_linear(a, w, b), atol=2e-3, rtol=2e-2)


def test_gemm_pair_strided_out_guard_bands(cuda_device):
    # fp16 output rows with a stride wider than N inside a guarded buffer: the
    # TMA stores write exactly the M x N window (M tail clipped).
    M, N, K, ldo, pad = 9000, 2048, 256, 2048 + 64, 8192
    a, w, b = operands(M, N, K, seed=47)
    buf = torch.full((M * ldo + 2 * pad,), 77.0, dtype=torch.float16, device="cuda")
    out = buf[pad:pad + M * ldo].view(M, ldo)[:, :N]
    tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "gelu", out=out)
    torch.cuda.synchronize()
    host = buf.cpu()
    assert torch.all(host[:pad] == 77.0) and torch.all(host[-pad:] == 77.0)
    assert torch.all(host[pad:pad + M * ldo].view(M, ldo)[:, N:] == 77.0)
    want = F.gelu(ref_linear(a, w, b), approximate="none")
    torch.testing.assert_close(out.float().cpu(), want, atol=2e-4, rtol=1e-3)


def test_gemm_pair_row_len(cuda_device):
    S, B, N, K = 256, 40, 2048, 256
    a, w, b = operands(B * S, N, K, seed=53)
    lengths = (torch.arange(B, dtype=torch.int32) * 37) % (S + 1)
    out = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "gelu", row_len=lengths.cuda(), seq_len=S)
    pad = (torch.arange(B * S) % S) >= lengths.repeat_interleave(S)
    got = out.float().cpu()
    assert torch.all(got[pad] == 0)
    want = F.gelu(ref_linear(a, w, b), approximate="none")
    torch.testing.assert_close(got[~pad], want[~pad], atol=2e-4, rtol=1e-3)


@pytest.mark.parametrize("row_len", [False, True])
def test_gemm_pair_resid_out_of_place(cuda_device, row_len):
    # sum_out != resid (or padded rows): the staged residual epilogue of the pair kernel
    S, B, N, K = 256, 64, 1024, 512
    M = B * S
    a, w, b = operands(M, N, K, seed=59)
    r = seeded(M, N, seed=60)
    rc = r.cuda()
    lengths = (torch.arange(B, dtype=torch.int32) * 53) % (S + 1)
    kw = dict(row_len=lengths.cuda(), seq_len=S) if row_len else {}
    s = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid", resid=rc, **kw)
    want = r + ref_linear(a, w, b)
    got = s.cpu()
    if row_len:
        pad = (torch.arange(M) % S) >= lengths.repeat_interleave(S)
        assert torch.all(got[pad] == 0)
        got, want = got[~pad], want[~pad]
    torch.testing.assert_close(got, want, atol=1e-4, rtol=1e-4)
    assert torch.equal(rc.cpu(), r)  # resid untouched


# ---- residual + LayerNorm over rows wider than a tile (tk_gemm_resid_ln) ----
# Per-row partial statistics of every 128-column slice in a workspace, the
# row's last slice normalising it. Same tolerances as the one-tile LN
# epilogue: fp32 sum 1e-4, fp16 LN output 2e-3/2e-2, fp32 LN output 1e-4.

WIDE_LN = [(65536, 1024, 1024), (4096, 1024, 4096), (300, 512, 200), (1, 768, 64), (5000, 2048, 256),
           (777, 4096, 512)]


def _ln_case(M, N, K, seed):
    a, w, b = operands(M, N, K, seed=seed)
    r = seeded(M, N, seed=seed + 3)
    g = seeded(N, seed=seed + 4, scale=0.5) + 1.0
    beta = seeded(N, seed=seed + 5, scale=0.5)
    return a, w, b, r, g, beta


@pytest.mark.parametrize("M,N,K", WIDE_LN)
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_gemm_resid_ln_wide_rows(cuda_device, M, N, K, out_dtype):
    a, w, b, r, g, beta = _ln_case(M, N, K, seed=M + N + K)
    s, h = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid_ln", resid=r.cuda(), ln_weight=g.cuda(),
                            ln_bias=beta.cuda(), eps=1e-5, out_dtype=out_dtype)
    want_s = r + ref_linear(a, w, b)
    torch.testing.assert_close(s.cpu(), want_s, atol=1e-4, rtol=1e-4)
    want_h = F.layer_norm(want_s, (N,), g, beta, 1e-5)
    tol = dict(atol=2e-3, rtol=2e-2) if out_dtype == torch.float16 else dict(atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(h.float().cpu(), want_h, **tol)


def test_gemm_resid_ln_in_place_workspace_reuse(cuda_device):
    """The residual stream updated in place, the same workspace across calls
    and across row counts (a larger call, then smaller ones, then the larger
    again): the counters every call leaves at zero keep it reusable."""
    N, K = 1024, 1024
    Mbig = 8192
    ws = torch.zeros(tk_linear.ln_workspace_bytes(Mbig, N), dtype=torch.uint8, device="cuda")
    for i, M in enumerate([Mbig, 1000, 4097, Mbig]):
        a, w, b, r, g, beta = _ln_case(M, N, K, seed=100 + i)
        res = r.cuda()
        h = torch.empty(M, N, dtype=torch.float16, device="cuda")
        tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid_ln", resid=res, sum_out=res, ln_weight=g.cuda(),
                         ln_bias=beta.cuda(), eps=1e-5, out=h, workspace=ws)
        want_s = r + ref_linear(a, w, b)
        torch.testing.assert_close(res.cpu(), want_s, atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(h.float().cpu(), F.layer_norm(want_s, (N,), g, beta, 1e-5), atol=2e-3, rtol=2e-2)
    torch.cuda.synchronize()
    count_bytes = (Mbig * 8 + 255) // 256 * 256
    assert int(ws[:count_bytes].view(torch.int64).abs().sum()) == 0  # every row state word back at zero


def test_gemm_resid_ln_row_len_and_large_mean(cuda_device):
    """Padded rows give s = 0 and h = 0; rows with a large common offset keep
    the centred statistics (a one-pass E[x^2] - E[x]^2 would lose them)."""
    S, B, N, K = 256, 24, 1024, 256
    M = B * S
    a, w, b, r, g, beta = _ln_case(M, N, K, seed=71)
    r = r + 300.0
    lengths = (torch.arange(B, dtype=torch.int32) * 41) % (S + 1)
    s, h = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid_ln", resid=r.cuda(), ln_weight=g.cuda(),
                            ln_bias=beta.cuda(), eps=1e-5, out_dtype=torch.float32, row_len=lengths.cuda(), seq_len=S)
    pad = (torch.arange(M) % S) >= lengths.repeat_interleave(S)
    got_s, got_h = s.cpu(), h.cpu()
    assert torch.all(got_s[pad] == 0) and torch.all(got_h[pad] == 0)
    want_s = r + ref_linear(a, w, b)
    torch.testing.assert_close(got_s[~pad], want_s[~pad], atol=1e-4, rtol=1e-4)
    want_h = F.layer_norm(want_s, (N,), g, beta, 1e-5)
    torch.testing.assert_close(got_h[~pad], want_h[~pad], atol=1e-3, rtol=1e-3)


def test_gemm_resid_ln_rejects_bad_workspace(cuda_device):
    import _tklib as tk

    M, N, K = 512, 1024, 256
    a, w, b, r, g, beta = _ln_case(M, N, K, seed=81)
    small = torch.zeros(tk_linear.ln_workspace_bytes(M, N) - 256, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError):
        tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid_ln", resid=r.cuda(), ln_weight=g.cuda(),
                         ln_bias=beta.cuda(), workspace=small)
    rc = tk.lib().tk_gemm_resid_ln(16, K, 16, K, 16, 16, N, 16, N, 16, 16, 1e-5, 16, 1, N, None, 0, M, N, K,
                                   None, 0, None)
    assert rc == -1 and b"workspace" in tk.lib().tk_last_error()


# ---- tile variants chosen through the measured table (tk_gemm_tiles_set) ----

@pytest.mark.parametrize("M,N,K,epi", [(16384, 3072, 1024, "bias"), (16384, 4096, 1024, "gelu"),
                                       (16384, 1024, 4096, "resid"), (512, 2048, 512, "gelu"), (777, 1536, 512, "bias")])
def test_every_tile_variant_matches_the_reference(cuda_device, M, N, K, epi):
    import _tklib as tk

    a, w, b = operands(M, N, K, seed=N + K)
    r = seeded(M, N, seed=5) if epi == "resid" else None
    want = ref_linear(a, w, b)
    if epi == "gelu":
        want = F.gelu(want, approximate="none")
    if epi == "resid":
        want = r + want
    code = tk_linear.EPILOGUES[epi]
    ran = set()
    try:
        for v in ("pair", "bn256", "bn128", "bn64"):
            tk.lib().tk_gemm_tiles_clear()
            tk.call("tk_gemm_tiles_set", M, N, K, code, tk.TILES[v])
            chosen = tk.lib().tk_gemm_tiles_chosen(M, N, K, code)
            if chosen != tk.TILES[v]:
                continue
            ran.add(v)
            if epi == "resid":
                out = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), "resid", resid=r.cuda())
                torch.testing.assert_close(out.cpu(), want, atol=1e-4, rtol=1e-4, msg=v)
            else:
                out = tk_linear.linear(a.cuda(), w.cuda(), b.cuda(), epi)
                tol = dict(atol=2e-4, rtol=1e-3) if epi == "gelu" else dict(atol=2e-3, rtol=2e-2)
                torch.testing.assert_close(out.float().cpu(), want, **tol, msg=v)
    finally:
        tk.lib().tk_gemm_tiles_clear()
    assert "bn64" in ran and ("pair" in ran) == (N % 256 == 0)
