"""ctypes binding of libtk_b200.so (the C ABI declared in include/tk_b200.h).

The library is built in-tree (``build.py``) and loaded from this directory.
There is no fallback: a missing library, a missing symbol, or a non-zero
status from any entry point raises ``TKError`` with the library's message.
"""

from __future__ import annotations

import ctypes
import os
import pathlib
from typing import Optional

import torch

HERE = pathlib.Path(__file__).resolve().parent
LIB_PATH = HERE / "libtk_b200.so"

TK_OK = 0
TK_F32, TK_F16 = 0, 1
EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESID, EPI_BIAS_RESID_LN = 0, 1, 2, 3
TILES = {"auto": 0, "pair": 1, "bn256": 2, "bn128": 3, "bn64": 4}

STATUS_NAMES = {
    -1: "TK_ERR_INVALID",
    -2: "TK_ERR_UNSUPPORTED",
    -3: "TK_ERR_LAUNCH",
    -4: "TK_ERR_TIMEOUT",
    -5: "TK_ERR_CUDA",
    -6: "TK_ERR_DEVICE",
}

# name -> (restype, argtypes); mirrors include/tk_b200.h
_P, _I, _I64, _F, _U64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64
SIGNATURES = {
    "tk_layernorm": (_I, [_P, _I, _I64, _P, _I, _I64, _P, _I64, _P, _P, _F, _P, _I, _I64, _P, _I64, _I64, _I64,
                          _P]),
    "tk_gemm": (_I, [_P, _I64, _P, _I64, _P, _I, _P, _I64, _P, _I64, _P, _P, _F, _P, _I, _I64, _P, _I64,
                     _I64, _I64, _I64, _P]),
    "tk_attn_fwd": (_I, [_P, _P, _P, _I64, _I64, _I64, _P, _I64, _I64, _I64, _I64, _I64, _F, _I, _P, _P]),
    "tk_layernorm_supported": (_I, [_I64]),
    "tk_attn_supported": (_I, [_I64]),
    "tk_check_device_errors": (_I, [_P]),
    "tk_set_wait_limit_ns": (_U64, [_U64]),
    "tk_set_programmatic_launch": (_I, [_I]),
    "tk_stack_small_supported": (_I, [_I64, _I64, _I64, _I64]),
    "tk_stack_small": (_I, [_P, _P, _P, _P, _P, _P, _F, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I, _F, _P]),
    "tk_selftest_wait_timeout": (_I, [_P]),
    "tk_gemm_resid_ln_workspace_bytes": (_I64, [_I64, _I64]),
    "tk_gemm_resid_ln_supported": (_I, [_I64, _I64, _I64]),
    "tk_gemm_resid_ln": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _P, _I64, _P, _P, _F, _P, _I, _I64, _P, _I64,
                              _I64, _I64, _I64, _P, _I64, _P]),
    "tk_gemm_resid_ln_static": (_I, [_P, _I64, _P, _I64, _P, _P, _I64, _P, _I64, _P, _P, _F, _P, _I, _I64, _P,
                                     _I64, _I64, _I64, _I64, _P]),
    "tk_gemm_tiles_set": (_I, [_I64, _I64, _I64, _I, _I]),
    "tk_gemm_tiles_clear": (_I, []),
    "tk_gemm_tiles_chosen": (_I, [_I64, _I64, _I64, _I]),
    "tk_peer_export": (_I, [_P, _P, ctypes.POINTER(ctypes.c_int64)]),
    "tk_peer_import": (_I, [_P, _I64, ctypes.POINTER(ctypes.c_void_p)]),
    "tk_peer_release": (_I, [_P]),
    "tk_copy_rows": (_I, [_P, _I64, _P, _I64, _I64, _I64, _P]),
    "tk_last_error": (ctypes.c_char_p, []),
    "tk_version": (ctypes.c_char_p, []),
}


class TKError(RuntimeError):
    """A libtk_b200 call returned a non-zero status."""

    def __init__(self, fn: str, status: int, message: str):
        self.status = status
        super().__init__(f"{fn}: {STATUS_NAMES.get(status, status)}: {message}")


_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is not built."""
    global _lib
    if _lib is None:
        path = pathlib.Path(os.environ.get("TK_B200_LIB", LIB_PATH))
        if not path.exists():
            raise TKError("load", -5, f"{path} not found; build it with transformer-kernel_b200/build.py")
        handle = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def call(name: str, *args) -> int:
    status = getattr(lib(), name)(*args)
    if status != TK_OK:
        raise TKError(name, status, lib().tk_last_error().decode(errors="replace"))
    return status


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return TK_F32
    if dt == torch.float16:
        return TK_F16
    raise TKError("dtype", -1, f"unsupported dtype {dt}; the kernels take float32 or float16")


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise TKError("device", -1, "libtk_b200 kernels take CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise TKError("device", -1, f"tensors on different devices: {dev} vs {t.device}")
    return dev


def check_device_errors(device: Optional[torch.device] = None) -> None:
    """Synchronise the current stream and raise if a kernel's bounded wait
    gave up since the last check."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(device):
        call("tk_check_device_errors", stream_handle(device))


def set_wait_limit_ns(ns: int) -> int:
    return int(lib().tk_set_wait_limit_ns(int(ns)))


def set_programmatic_launch(enable: bool) -> bool:
    """Launch later launch-bound (small) kernels with programmatic dependent
    launch (default on; large kernels always launch plainly). Returns the
    previous setting."""
    return bool(lib().tk_set_programmatic_launch(1 if enable else 0))


def version() -> str:
    return lib().tk_version().decode()


def peer_export(t: torch.Tensor) -> tuple:
    """(64-byte handle, byte offset) naming the device allocation of ``t``,
    for ``peer_import`` in another process of the same node."""
    handle = ctypes.create_string_buffer(64)
    offset = ctypes.c_int64(0)
    call("tk_peer_export", t.data_ptr(), handle, ctypes.byref(offset))
    return handle.raw, int(offset.value)


def peer_import(handle: bytes, offset: int) -> int:
    """Device address, in this process, of a pointer another process exported."""
    if len(handle) != 64:
        raise TKError("tk_peer_import", -1, "handle must be the 64 bytes tk_peer_export wrote")
    ptr = ctypes.c_void_p(0)
    call("tk_peer_import", ctypes.create_string_buffer(handle, 64), int(offset), ctypes.byref(ptr))
    return int(ptr.value)


def peer_release(ptr: int) -> None:
    call("tk_peer_release", ptr)


def copy_rows(dst: int, dst_ld: int, src: int, src_ld: int, row_bytes: int, rows: int, stream: int) -> None:
    """Stream-ordered copy of ``rows`` rows of ``row_bytes`` between device
    addresses (either may be an imported peer address)."""
    call("tk_copy_rows", dst, dst_ld, src, src_ld, row_bytes, rows, stream)
