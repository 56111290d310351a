"""CPU checks of the C ABI: the library loads, exports every entry point
that include/tk_b200.h declares, and rejects bad arguments on the host
before touching a device (so these run without a GPU)."""

from __future__ import annotations

import ctypes
import pathlib
import re

import pytest

import _tklib as tk

HEADER = pathlib.Path(__file__).resolve().parents[1] / "include" / "tk_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TK_API\s+[\w\s\*]+?\b(tk_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"tk_layernorm", "tk_gemm", "tk_attn_fwd", "tk_check_device_errors"} <= set(names)


def test_library_exports_every_declared_symbol():
    lib = tk.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    # the ctypes table covers every declared symbol too
    assert set(declared_symbols()) <= set(tk.SIGNATURES)


def test_version_and_probes():
    lib = tk.lib()
    assert b"sm_100a" in lib.tk_version()
    assert lib.tk_attn_supported(32) == 1 and lib.tk_attn_supported(64) == 1
    assert lib.tk_attn_supported(8) == 1 and lib.tk_attn_supported(16) == 1
    assert lib.tk_attn_supported(128) == 1 and lib.tk_attn_supported(256) == 1
    assert lib.tk_attn_supported(96) == 0 and lib.tk_attn_supported(24) == 0
    assert lib.tk_layernorm_supported(1) == 1 and lib.tk_layernorm_supported(8192) == 1
    assert lib.tk_layernorm_supported(8193) == 0 and lib.tk_layernorm_supported(0) == 0


def test_wait_limit_roundtrip():
    old = tk.set_wait_limit_ns(12345)
    assert tk.set_wait_limit_ns(old) == 12345


@pytest.mark.parametrize(
    "args, status",
    [
        # null operands
        (dict(A=None), -1),
        # N not a multiple of 32
        (dict(N=100), -2),
        # misaligned row stride
        (dict(lda=1001), -1),
        # fused LN on a width that does not fit one tile
        (dict(epi=3, N=512), -2),
    ],
)
def test_gemm_rejects_bad_arguments_on_host(args, status):
    lib = tk.lib()
    a = dict(A=16, lda=1024, W=16, ldw=1024, bias=16, epi=0, M=128, N=256, K=1024)
    a.update(args)
    rc = lib.tk_gemm(a["A"], a["lda"], a["W"], a["ldw"], a["bias"], a["epi"], 16, a["N"], 16, a["N"], 16, 16,
                     1e-5, 16, 1, 1024, None, 0, a["M"], a["N"], a["K"], None)
    assert rc == status
    assert lib.tk_last_error() != b""


def test_attention_rejects_unsupported_head_dim_on_host():
    lib = tk.lib()
    rc = lib.tk_attn_fwd(16, 16, 16, 3 * 96 * 384, 96, 3 * 384, 16, 384, 1, 128, 4, 96, 0.1, 1, None, None)
    assert rc == -2 and b"head_dim" in lib.tk_last_error()


def test_layernorm_rejects_bad_arguments_on_host():
    lib = tk.lib()
    assert lib.tk_layernorm(16, 0, 64, None, 0, 0, None, 0, 16, 16, 1e-5, 16, 1, 64, None, 0, 4, 9000, None) == -2
    assert lib.tk_layernorm(None, 0, 64, None, 0, 0, None, 0, 16, 16, 1e-5, 16, 1, 64, None, 0, 4, 64, None) == -1
    # a copy-through sum_out whose row stride is shorter than a row
    assert lib.tk_layernorm(16, 0, 64, None, 0, 0, 16, 32, 16, 16, 1e-5, 16, 1, 64, None, 0, 4, 64, None) == -1


def test_python_wrappers_refuse_cpu_tensors():
    import torch

    import fused_kernels

    x = torch.randn(4, 64)
    with pytest.raises(tk.TKError):
        fused_kernels.ln_fwd(x, torch.ones(64), torch.zeros(64), 1e-5)
    assert not fused_kernels.can_fuse(x)


def test_resid_ln_workspace_and_support_on_host():
    lib = tk.lib()
    # one tile holds rows of 64/128/256: no workspace
    assert lib.tk_gemm_resid_ln_workspace_bytes(65536, 256) == 0
    # state words [M] u64 + partials [M, N/128] float2, each 256-byte aligned
    assert lib.tk_gemm_resid_ln_workspace_bytes(65536, 1024) == 65536 * 8 + 65536 * 8 * 8
    assert lib.tk_gemm_resid_ln_workspace_bytes(1000, 512) == 8192 + 32000
    assert lib.tk_gemm_resid_ln_supported(65536, 1024, 4096) == 1
    assert lib.tk_gemm_resid_ln_supported(65536, 640, 4096) == 0   # not a multiple of 256
    assert lib.tk_gemm_resid_ln_supported(65536, 8192, 4096) == 0  # above 4096
    assert lib.tk_gemm_resid_ln_supported(65536, 1024, 12) == 0    # K % 8
    # refused before any launch: unsupported width, missing workspace
    assert lib.tk_gemm_resid_ln(16, 64, 16, 64, 16, 16, 640, 16, 640, 16, 16, 1e-5, 16, 1, 640, None, 0, 8, 640, 64,
                                16, 4096, None) == -2
    assert lib.tk_gemm_resid_ln(16, 64, 16, 64, 16, 16, 1024, 16, 1024, 16, 16, 1e-5, 16, 1, 1024, None, 0, 8, 1024,
                                64, None, 0, None) == -1
