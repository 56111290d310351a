"""Error bounds of the device-side approximations, restated on the CPU.

The attention softmax takes a quarter of its exponentials on the FMA pipe
(csrc/tk_attn.cuh exp2_fma_pair: Cody-Waite reduction plus a cubic
fitted for minimum relative error), and the FFN-in GEMM epilogue computes the
erf GELU by Abramowitz & Stegun 7.1.28 (csrc/tk_gemm.cuh gelu_erf2). Both are
restated here in float32 steps, with the constants parsed from the shipped
headers, and compared with double-precision references: relative error of
2^x below 8e-5 (under fp16's 2^-11 rounding of P), absolute GELU error below
1e-6 (the reference computes the exact erf GELU in fp32,
src/torch_transformer_benchmark.py:141). The device instructions themselves
(rcp.approx, f32x2 FMA) are exercised by the GPU parity tests."""

from __future__ import annotations

import math
import pathlib
import re

import numpy as np

CSRC = pathlib.Path(__file__).resolve().parents[1] / "transformer-kernel_b200" / "csrc"
f32 = np.float32


def _constants(header: str, names):
    text = (CSRC / header).read_text()
    out = {}
    for name in names:
        m = re.search(rf"\b{name}\s*=\s*([0-9.eE+-]+)f", text)
        assert m, f"{name} not found in {header}"
        out[name] = f32(float(m.group(1)))
    return out


def _fma(a, b, c):
    # float32 fused multiply-add: the float32 product is exact in float64
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(f32)


def exp2_fma_cpu(x: np.ndarray) -> np.ndarray:
    c = _constants("tk_attn.cuh", ["kC0", "kC1", "kC2", "kC3", "kRound"])
    x = np.maximum(x.astype(f32), f32(-126.0))
    t = (x + c["kRound"]).astype(f32)
    f = (x - (t - c["kRound"]).astype(f32)).astype(f32)
    q = _fma(_fma(_fma(np.full_like(f, c["kC3"]), f, np.full_like(f, c["kC2"])), f, np.full_like(f, c["kC1"])),
             f, np.full_like(f, c["kC0"]))
    bits = q.view(np.int32) + (t.view(np.int32) << 23)
    return bits.astype(np.int32).view(f32)


def gelu_erf_cpu(v: np.ndarray) -> np.ndarray:
    a = _constants("tk_gemm.cuh", ["kA1", "kA2", "kA3", "kA4", "kA5", "kA6"])
    inv_sqrt2 = f32(0.70710678118654752)
    v = v.astype(f32)
    z = (np.abs(v) * inv_sqrt2).astype(f32)
    q = _fma(z, np.full_like(z, a["kA6"]), np.full_like(z, a["kA5"]))
    for k in ("kA4", "kA3", "kA2", "kA1"):
        q = _fma(q, z, np.full_like(z, a[k]))
    q = _fma(q, z, np.ones_like(z))
    with np.errstate(over="ignore"):
        for _ in range(4):
            q = (q * q).astype(f32)
        r = (f32(1.0) / q).astype(f32)
    neg_half_abs = (z * -inv_sqrt2).astype(f32)
    return _fma(neg_half_abs, r, np.maximum(v, f32(0.0)))


def test_exp2_fma_relative_error():
    x = np.linspace(-30.0, 8.0, 2_000_003, dtype=np.float64).astype(f32)
    got = exp2_fma_cpu(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got - want) / want
    assert rel.max() < 8e-5, rel.max()


def test_exp2_fma_far_below_range_is_tiny():
    x = np.array([-126.0, -200.0, -1e4, -3.4e38], dtype=f32)
    got = exp2_fma_cpu(x)
    assert np.all(np.isfinite(got)) and np.all(got >= 0) and np.all(got <= 2.0 ** -125)
    # fp16 P: everything below 2^-25 rounds to zero
    assert np.all(got.astype(np.float16) == 0)


def test_gelu_erf_absolute_error():
    x = np.concatenate([np.linspace(-12.0, 12.0, 1_200_001), [-1e4, -60.0, 60.0, 1e4]]).astype(f32)
    got = gelu_erf_cpu(x).astype(np.float64)
    xd = x.astype(np.float64)
    want = 0.5 * xd * (1.0 + np.vectorize(math.erf)(xd / math.sqrt(2.0)))
    err = np.abs(got - want)
    assert err.max() < 1e-6, err.max()
    # large |x|: the power overflows, r = 0, GELU(x) = max(x, 0)
    assert got[-4] == 0.0 and got[-1] == 1e4
