"""ctypes binding of ``libtllm_sm100a.so`` (the C ABI declared in ``include/tllm_sm100.h``).

The library is built in-tree (``python -m tritonllmcompiler_b200.build``). There is no
fallback: when the library is missing or fails to load, every operator raises.
"""
from __future__ import annotations

import contextlib
import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libtllm_sm100a.so")

DTYPE_CODES = {torch.float16: 0, torch.bfloat16: 1}

_c_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64

# name -> (restype, argtypes); mirrors include/tllm_sm100.h.
SIGNATURES = {
    "tllm_version": (ctypes.c_char_p, []),
    "tllm_last_error": (ctypes.c_char_p, []),
    "tllm_debug_status": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int)]),
    "tllm_selftest_bounded_wait": (ctypes.c_int, [_vp]),
    "tllm_flash_attn_fwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _c_i64p, _c_i64p, _c_i64p, _c_i64p,
         ctypes.c_float, ctypes.c_int, ctypes.c_int, _vp],
    ),
    "tllm_flash_attn_fwd_variant": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _c_i64p, _c_i64p, _c_i64p, _c_i64p,
         ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp],
    ),
    "tllm_paged_attn_workspace_size": (ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64]),
    "tllm_paged_attn_decode": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _i64, _i64, _i64, _i64, _i64, _i64,
         _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, ctypes.c_float, ctypes.c_int, _vp],
    ),
    "tllm_paged_attn_decode_noalloc": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64,
         _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, ctypes.c_float, ctypes.c_int, _vp],
    ),
    "tllm_rmsnorm_rope": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _c_i64p, _i64, _c_i64p, _c_i64p,
         _c_i64p, ctypes.c_float, ctypes.c_int, _vp],
    ),
    "tllm_swiglu_colshard": (
        ctypes.c_int,
        [_vp, _vp, _vp, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _i64, _i64, _i64, _i64,
         _i64, _i64, _i64, _i64, ctypes.c_int, _vp],
    ),
    "tllm_swiglu_colshard_peers": (
        ctypes.c_int,
        [_vp, _vp, _vp, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
         ctypes.c_int, ctypes.c_int, _vp, ctypes.c_uint32, _i64, _i64, _i64, _i64, _i64, _i64,
         _i64, ctypes.c_int, ctypes.c_int, _vp],
    ),
    "tllm_swiglu_colshard_multicast": (
        ctypes.c_int,
        [_vp, _vp, _vp, ctypes.POINTER(ctypes.c_void_p), _vp, ctypes.POINTER(ctypes.c_void_p),
         ctypes.c_int, ctypes.c_int, _vp, ctypes.c_uint32, _i64, _i64, _i64, _i64, _i64, _i64,
         _i64, ctypes.c_int, _vp],
    ),
    "tllm_ipc_get_handle": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(ctypes.c_uint64)]),
    "tllm_ipc_open": (ctypes.c_int, [_vp, ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p),
                                     ctypes.POINTER(ctypes.c_void_p)]),
    "tllm_ipc_close": (ctypes.c_int, [_vp]),
    "tllm_copy2d_async": (ctypes.c_int, [_vp, ctypes.c_size_t, _vp, ctypes.c_size_t, ctypes.c_size_t,
                                         ctypes.c_size_t, _vp]),
    "tllm_paged_kv_append": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
         _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, ctypes.c_int, _vp],
    ),
    "tllm_paged_kv_append_rope": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
         _i64, _i64, _i64, _i64, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, ctypes.c_float,
         ctypes.c_int, _vp],
    ),
    "tllm_paged_prefill_workspace_size": (ctypes.c_size_t, [_i64, _i64, _i64, _i64, _i64, _i64, _i64]),
    "tllm_paged_prefill": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _i64, _i64, _i64, _i64, _i64, _i64,
         _i64, _i64, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, ctypes.c_float, ctypes.c_int,
         ctypes.c_int, _vp],
    ),
    "tllm_flash_attn_varlen_fwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
         _c_i64p, _c_i64p, _c_i64p, _c_i64p, ctypes.c_float, ctypes.c_int, ctypes.c_int, _vp],
    ),
    "tllm_flash_attn_fwd_lse": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _c_i64p, _c_i64p, _c_i64p,
         _c_i64p, ctypes.c_float, ctypes.c_int, ctypes.c_int, _vp],
    ),
    "tllm_flash_attn_bwd_workspace_size": (ctypes.c_size_t, [_i64, _i64, _i64, _i64]),
    "tllm_flash_attn_bwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _i64, _i64, _i64,
         _i64, _i64, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p, _c_i64p,
         ctypes.c_float, ctypes.c_int, ctypes.c_int, _vp],
    ),
    "tllm_swiglu_fp8": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float,
         ctypes.c_float, ctypes.c_float, ctypes.c_int, _vp],
    ),
    "tllm_swiglu_fp8_variant": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_float,
         ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int, _vp],
    ),
    "tllm_flash_attn_fp8_fwd": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _c_i64p, _c_i64p, _c_i64p, _c_i64p,
         ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int,
         ctypes.c_int, _vp],
    ),
    "tllm_qkv_norm_rope": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
         _i64, _i64, _i64, ctypes.c_float, ctypes.c_int, _vp],
    ),
    "tllm_swiglu_variant": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_int, ctypes.c_int, _vp],
    ),
    "tllm_swiglu": (
        ctypes.c_int,
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, ctypes.c_int, _vp],
    ),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads (once) and returns the extension; raises RuntimeError if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m tritonllmcompiler_b200.build`"
                    " (the operators have no non-CUDA implementation)"
                )
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int) -> None:
    """Raises RuntimeError with the library's message for a non-zero status."""
    if rc != 0:
        msg = load().tllm_last_error().decode("utf-8", "replace")
        raise RuntimeError(f"libtllm_sm100a: {msg} (status {rc})")


def strides(t: torch.Tensor, n: int | None = None):
    """Element strides of ``t`` as a ctypes int64 array."""
    s = t.stride()
    if n is not None:
        s = tuple(s[:n])
    return (ctypes.c_int64 * len(s))(*s)


def ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t: torch.Tensor) -> int:
    """The current CUDA stream of ``t``'s device, as a raw handle."""
    if _raw_stream is not None:
        return _raw_stream(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


def on_device(t: torch.Tensor):
    """Context making ``t``'s device current for the library call (the C entry points work on
    the current device); a no-op when it already is, which is the common case and saves the
    cost of switching devices on every call."""
    if t.device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(t.device)


def debug_status() -> int:
    """Reads and clears the device error word (synchronises the current device)."""
    out = ctypes.c_int(0)
    check(load().tllm_debug_status(ctypes.byref(out)))
    return out.value
