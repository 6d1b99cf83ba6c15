"""ctypes binding of libjishui_b200.so (the C ABI declared in include/jishui_b200.h).

The library is loaded from the package directory; there is no fallback: if the
shared object is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import threading
from ctypes import c_float, c_int, c_int64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libjishui_b200.so"

_P = c_void_p
_SIGNATURES: dict[str, tuple] = {
    "jx_version": (c_int, []),
    "jx_last_error": (ctypes.c_char_p, []),
    "jx_launch_count": (c_int64, []),
    "jx_device_status": (c_int, [ctypes.POINTER(c_int), c_int]),
    "jx_set_sm_reserve": (c_int, [c_int]),
    "jx_rmsnorm_fwd": (c_int, [_P, _P, _P, _P, _P, _P, c_int64, c_int, c_float, _P]),
    "jx_rmsnorm_bwd_parts": (c_int, [c_int64]),
    "jx_rmsnorm_bwd": (c_int, [_P, _P, _P, _P, _P, _P, _P, c_int64, c_int, _P]),
    "jx_rmsnorm_dgamma_reduce": (c_int, [_P, c_int, c_int, _P, c_int, _P]),
    "jx_layernorm_fwd": (c_int, [_P, _P, _P, _P, _P, _P, c_int64, c_int, c_float, _P]),
    "jx_layernorm_bwd": (c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, c_int64, c_int, _P]),
    "jx_attn_decode_workspace_bytes": (c_int64, [c_int, c_int, c_int]),
    "jx_attn_decode": (c_int, [_P, c_int64, _P, _P, c_int64, c_int64, c_int, c_int, _P, c_int, c_int, c_float, _P,
                               _P, c_int64, _P]),
    "jx_pack_rows": (c_int, [_P, c_int64, _P, _P, c_int, c_int, _P, _P]),
    "jx_rmsnorm_bwd_noalloc": (c_int, [_P, _P, _P, _P, _P, _P, _P, c_int, c_int64, c_int, _P]),
    "jx_embed_fwd": (c_int, [_P, c_int64, _P, c_int64, c_int, _P, _P]),
    "jx_embed_bwd": (c_int, [_P, c_int64, _P, c_int64, c_int, _P, _P]),
    "jx_gemm_f16": (c_int, [_P, c_int64, c_int, _P, c_int64, c_int, c_int, c_int, c_int, _P, c_int64, _P, c_int64, _P]),
    "jx_gemm_qkv_rope": (c_int, [_P, c_int64, _P, c_int, c_int, c_int, _P, c_int64, _P, _P, c_int, c_int, _P]),
    "jx_gemm_swiglu_fwd": (c_int, [_P, c_int64, _P, c_int, c_int, c_int, _P, _P, _P, c_int64, _P]),
    "jx_gemm_swiglu_bwd": (c_int, [_P, c_int64, _P, c_int, c_int, c_int, _P, _P, c_int64, _P, c_int64, _P]),
    "jx_gemm_wgrad_workspace_bytes": (c_int64, [c_int, c_int, c_int]),
    "jx_gemm_set_mode": (c_int, [c_int]),
    "jx_gemm_wait_test": (c_int, [_P, _P, _P, c_int64, _P]),
    "jx_gemm_wgrad": (c_int, [_P, c_int64, _P, c_int64, c_int, c_int, c_int, _P, c_int64, c_int, c_int, _P, _P]),
    "jx_attn_fwd_workspace_bytes": (c_int64, [c_int, c_int, c_int, c_int]),
    "jx_attn_fwd": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_float, _P]),
    "jx_attn_bwd_workspace_bytes": (c_int64, [c_int, c_int, c_int, c_int]),
    "jx_attn_bwd": (c_int, [_P, _P, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_float, _P, _P, _P]),
    "jx_ce_fwd": (c_int, [_P, c_int64, c_int, c_int64, _P, c_int64, _P, _P, _P]),
    "jx_gemm_f16_ce_parts": (c_int, [_P, c_int64, _P, c_int64, c_int, c_int, c_int, _P, c_int64, _P, _P]),
    "jx_ce_fwd_parts": (c_int, [_P, c_int, _P, c_int64, c_int, c_int64, _P, c_int64, _P, _P, _P]),
    "jx_ce_loss": (c_int, [_P, _P, c_int64, c_int64, _P, c_int, _P]),
    "jx_ce_bwd": (c_int, [_P, c_int64, c_int, c_int64, _P, c_int64, _P, _P, _P, _P]),
    "jx_grad_stats_parts": (c_int, [c_int64]),
    "jx_grad_stats": (c_int, [_P, c_int, c_int64, _P, _P, _P, _P, _P]),
    "jx_grad_finalize": (c_int, [_P, c_int, c_float, _P, _P]),
    "jx_adamw_step": (c_int, [_P, _P, c_int, _P, _P, _P, c_int64, _P, _P, _P, _P, c_float, c_float, c_float,
                              c_float, c_float, _P]),
    "jx_scaler_update": (c_int, [_P, _P, _P, c_float, c_float, c_int, _P]),
    "jx_cast_f32_f16": (c_int, [_P, _P, c_int64, _P]),
    "jx_transpose_f16": (c_int, [_P, _P, c_int64, c_int64, _P]),
}

EXPORTED = tuple(_SIGNATURES)

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads the shared library once and binds every declared symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m midstream_llm_b200.build` "
                                   "(the CUDA kernels have no fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class JxError(RuntimeError):
    pass


def call(name: str, *args) -> None:
    """Invokes an entry point; a non-zero status raises with the library's error text."""
    rc = getattr(load(), name)(*args)
    if rc != 0:
        msg = load().jx_last_error().decode(errors="replace")
        raise JxError(f"{name} failed ({rc}): {msg}")


def query(name: str, *args):
    return getattr(load(), name)(*args)


def launch_count() -> int:
    """Kernels launched by libjishui_b200.so so far in this process."""
    return int(load().jx_launch_count())


def device_status(clear: bool = True) -> int:
    v = c_int(0)
    call("jx_device_status", ctypes.byref(v), int(clear))
    return v.value
