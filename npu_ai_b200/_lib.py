"""ctypes binding of libnpub200.so (the C ABI declared in include/npu_b200.h).

There is no fallback: if the library is missing or does not load, every call raises. Errors from the library
map onto the reference's exception types: an invalid request -> ValueError (the reference raises ValueError for
shapes it cannot take, npu/xdna1_gemm.py:227-229, :532-533), everything else -> RuntimeError (a failed NPU
command raises RuntimeError, npu/xdna1_program.py:475-479).
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libnpub200.so")
TORCH_OPS_PATH = os.path.join(HERE, "libnpub200_torch.so")

OK, EINVAL, ECUDA, EUNSUPPORTED, EDEVICE = 0, -1, -2, -3, -4
DTYPE_BF16, DTYPE_F32 = 0, 1

_c_i64 = ctypes.c_int64
_c_p = ctypes.c_void_p
_SIGNATURES = {
    "npub200_version": (ctypes.c_int, []),
    "npub200_last_error": (ctypes.c_char_p, []),
    "npub200_device_sms": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "npub200_weight_register": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, ctypes.POINTER(_c_i64)]),
    "npub200_weight_release": (ctypes.c_int, [_c_i64]),
    "npub200_gemm_workspace_size": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, ctypes.c_int,
                                                   ctypes.POINTER(ctypes.c_size_t)]),
    "npub200_gemm_plan": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                         ctypes.POINTER(ctypes.c_int)]),
    "npub200_gemm": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_p, ctypes.c_int, _c_p,
                                    _c_i64, ctypes.c_int, _c_p, ctypes.c_size_t, ctypes.c_int, _c_p]),
    "npub200_gemm_geglu": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_p, ctypes.c_int,
                                          _c_p, _c_i64, ctypes.c_int, _c_p, ctypes.c_size_t, ctypes.c_int, _c_p]),
    "npub200_conv3x3": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_p, ctypes.c_int, _c_i64,
                                       _c_p, _c_i64, _c_p, _c_i64, ctypes.c_int, _c_p, ctypes.c_size_t, ctypes.c_int,
                                       _c_p]),
    "npub200_conv3x3_workspace_size": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int,
                                                      ctypes.POINTER(ctypes.c_size_t)]),
    "npub200_group_norm": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, ctypes.c_float, ctypes.c_int,
                                          _c_p, _c_p, _c_p]),
    "npub200_group_norm_scratch_size": (ctypes.c_int, [_c_i64, _c_i64, ctypes.POINTER(ctypes.c_size_t)]),
    "npub200_layer_norm": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_p, ctypes.c_int, ctypes.c_float, _c_p,
                                          _c_i64, _c_p]),
    "npub200_upsample_nearest2x": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p]),
    "npub200_concat_channels": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64,
                                               _c_p]),
    "npub200_gemm_residual": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_p, ctypes.c_int,
                                             _c_p, _c_i64, _c_p, _c_i64, ctypes.c_int, _c_p, ctypes.c_size_t,
                                             ctypes.c_int, _c_p]),
    "npub200_gemm_noalloc": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_p, ctypes.c_int,
                                            _c_p, _c_i64, ctypes.c_int, ctypes.c_int, _c_p]),
    "npub200_gemm_w": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, ctypes.c_int, _c_p, _c_i64,
                                      ctypes.c_int, _c_p, ctypes.c_size_t, ctypes.c_int, _c_p]),
    "npub200_attention": (ctypes.c_int, [_c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64,
                                         _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_i64, _c_i64,
                                         _c_i64, _c_i64, _c_i64, ctypes.c_float, ctypes.c_int, _c_p]),
    "npub200_status_read": (ctypes.c_int, [_c_p, ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]),
    "npub200_set_wait_timeout_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "npub200_set_debug_flags": (ctypes.c_int, [ctypes.c_uint32]),
}

_lib = None
_lock = threading.Lock()


class KernelLibraryMissing(RuntimeError):
    """libnpub200.so is not built or cannot be loaded; the hot path has no CPU fallback."""


def load() -> ctypes.CDLL:
    """The loaded library (loaded once per process)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise KernelLibraryMissing(
                    f"{LIB_PATH} is missing: build it with `python -m npu_ai_b200.build` (there is no CPU fallback)")
            try:
                lib = ctypes.CDLL(LIB_PATH)
            except OSError as e:
                raise KernelLibraryMissing(f"cannot load {LIB_PATH}: {e}") from e
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


_ops = None


def torch_ops():
    """torch.ops.npub200: the GEMM and the fused attention as torch operators (libnpub200_torch.so, a thin
    TORCH_LIBRARY layer over this same C ABI, running on torch's current CUDA stream), or None when that library
    is not built. Loads libnpub200.so first, so both bindings share one instance of the kernel library."""
    global _ops
    if _ops is not None:
        return _ops
    load()
    if not os.path.exists(TORCH_OPS_PATH):
        return None
    with _lock:
        if _ops is None:
            import torch
            torch.ops.load_library(TORCH_OPS_PATH)
            _ops = torch.ops.npub200
    return _ops


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> str:
    msg = load().npub200_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(rc: int, what: str) -> None:
    """Raise the reference's exception type for a failing library call."""
    if rc == OK:
        return
    msg = last_error()
    if rc == EINVAL:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what} failed ({rc}): {msg}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)
