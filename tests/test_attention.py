"""tk_attn_fwd parity (GPU) against the baseline-order reference
(src/test_triton_kernels.py:125-216): fp32 scores scaled after q.k, -inf
mask, fp32 softmax, PV. Tolerance atol 2e-3 / rtol 2e-2 as in the
reference's attention tests. Shapes follow the reference's list restricted
to the head dims these kernels take (8, 16, 32, 64, 128, 256; 8 runs
zero-padded to 16, 128 and 256 the chunked kernel); others must be refused."""

from __future__ import annotations

import pytest
import torch

import _tklib as tk
import kernels
from oracle import attention_reference

pytestmark = pytest.mark.gpu


def seeded(*shape, seed=0, dtype=torch.float16):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype)


SHAPES = [(2, 4, 128, 32), (2, 4, 96, 32), (1, 2, 128, 64), (1, 4, 32, 64), (2, 3, 384, 64), (1, 2, 1000, 64),
          (3, 2, 257, 32), (2, 4, 128, 16), (1, 3, 300, 16), (2, 4, 128, 8), (1, 16, 200, 8),
          (2, 1, 128, 128), (1, 2, 520, 128), (2, 2, 128, 256), (1, 1, 300, 256)]


def run(q, k, v, causal, kv_len=None):
    out = kernels.flash_attention(q.cuda(), k.cuda(), v.cuda(), q.shape[-1] ** -0.5, causal,
                                  kv_len=None if kv_len is None else kv_len.cuda())
    return out.float().cpu()


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "b{}h{}s{}d{}".format(*s))
@pytest.mark.parametrize("causal", [True, False], ids=["causal", "full"])
def test_attention_matches_reference(cuda_device, shape, causal):
    b, h, s, hd = shape
    q, k, v = seeded(b, h, s, hd, seed=1), seeded(b, h, s, hd, seed=2), seeded(b, h, s, hd, seed=3)
    out = run(q, k, v, causal)
    ref = attention_reference(q, k, v, hd ** -0.5, causal)
    assert out.shape == (b, s, h * hd)
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-2)


def test_attention_strided_qkv_views(cuda_device):
    """The views the model passes: permuted slices of a fused [B, S, 3, H, hd]."""
    b, h, s, hd = 2, 4, 200, 64
    qkv = seeded(b, s, 3, h, hd, seed=42).cuda()
    q, k, v = qkv.permute(2, 0, 3, 1, 4).unbind(0)
    assert not q.is_contiguous()
    out = kernels.flash_attention(q, k, v, hd ** -0.5, True).float().cpu()
    ref = attention_reference(q.cpu().contiguous(), k.cpu().contiguous(), v.cpu().contiguous(), hd ** -0.5, True)
    torch.testing.assert_close(out, ref, atol=2e-3, rtol=2e-2)


def test_attention_output_layout(cuda_device):
    b, h, s, hd = 1, 2, 64, 64
    q, k, v = seeded(b, h, s, hd, seed=5), seeded(b, h, s, hd, seed=6), seeded(b, h, s, hd, seed=7)
    out = kernels.flash_attention(q.cuda(), k.cuda(), v.cuda(), hd ** -0.5, True)
    assert out.stride() == (s * h * hd, h * hd, 1)


@pytest.mark.parametrize("s", [32, 33, 64, 100, 129, 255])
def test_attention_ragged_sequence_lengths(cuda_device, s):
    b, h, hd = 1, 2, 32
    q, k, v = seeded(b, h, s, hd, seed=s), seeded(b, h, s, hd, seed=s + 1), seeded(b, h, s, hd, seed=s + 2)
    torch.testing.assert_close(run(q, k, v, True), attention_reference(q, k, v, hd ** -0.5, True),
                               atol=2e-3, rtol=2e-2)


@pytest.mark.parametrize("causal", [True, False])
def test_attention_kv_len_prefix_mask(cuda_device, causal):
    b, h, s, hd = 4, 2, 300, 64
    q, k, v = seeded(b, h, s, hd, seed=61), seeded(b, h, s, hd, seed=62), seeded(b, h, s, hd, seed=63)
    kv_len = torch.tensor([300, 1, 129, 200], dtype=torch.int32)
    out = run(q, k, v, causal, kv_len)
    ref = attention_reference(q, k, v, hd ** -0.5, causal, kv_len=kv_len)
    # rows whose every key is masked are NaN in the reference; compare the rest
    valid = torch.isfinite(ref)
    torch.testing.assert_close(out[valid], ref[valid], atol=2e-3, rtol=2e-2)


def test_attention_large_logits_stay_finite(cuda_device):
    """Scores spanning > 2^8 in the exponent exercise the lazy-rescale path."""
    b, h, s, hd = 1, 2, 512, 64
    q = seeded(b, h, s, hd, seed=71, dtype=torch.float32) * 4
    k = seeded(b, h, s, hd, seed=72, dtype=torch.float32) * 4
    v = seeded(b, h, s, hd, seed=73)
    q, k = q.half(), k.half()
    for causal in (True, False):
        out = run(q, k, v, causal)
        assert torch.isfinite(out).all()
        torch.testing.assert_close(out, attention_reference(q, k, v, hd ** -0.5, causal), atol=2e-3, rtol=2e-2)


def test_supported_probes(cuda_device):
    dev = torch.device("cuda")
    assert kernels.attention_supported(32, torch.float16, dev)
    assert kernels.attention_supported(64, torch.float16, dev)
    assert kernels.attention_supported(8, torch.float16, dev)
    assert kernels.attention_supported(16, torch.float16, dev)
    assert kernels.attention_supported(128, torch.float16, dev)
    assert kernels.attention_supported(256, torch.float16, dev)
    assert not kernels.attention_supported(96, torch.float16, dev)
    assert not kernels.attention_supported(64, torch.float32, dev)
    q = seeded(1, 1, 64, 96).cuda()
    with pytest.raises(tk.TKError):
        kernels.flash_attention(q, q, q, 0.1, True)
