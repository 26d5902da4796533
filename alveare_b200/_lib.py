"""ctypes binding of the C ABI in ``include/alveare_b200.h``.

This is the same binding a maintainer of the reference would add to its
Python runtime: plain pointers, sizes and int status codes.  The product path
fails loudly when the native library is missing; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libalveare_b200.so")

STATUS = {
    0: "ALV_OK",
    1: "ALV_ERR_ARG",
    2: "ALV_ERR_HANDLE",
    3: "ALV_ERR_SHAPE",
    4: "ALV_ERR_CUDA",
    5: "ALV_ERR_TIMEOUT",
    6: "ALV_ERR_UNSUPPORTED",
    7: "ALV_ERR_NO_DEVICE",
}
F32, BF16 = 0, 1
ACT_GELU, ACT_SILU = 0, 1

_c = ctypes
_vp = _c.c_void_p
_i = _c.c_int
_u32 = _c.c_uint32
_sz = _c.c_size_t

# name -> (restype, argtypes); one entry per function declared in the header.
IPC_BLOB_BYTES = 128  # ALV_IPC_BLOB_BYTES

SIGNATURES = {
    "alv_version": (_i, []),
    "alv_ctx_create": (_i, [_i, _c.POINTER(_vp)]),
    "alv_ctx_destroy": (_i, [_vp]),
    "alv_last_error": (_c.c_char_p, [_vp]),
    "alv_sync_status": (_i, [_vp, _vp]),
    "alv_q4_quantize": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "alv_gemv_weight_create": (_i, [_vp, _i, _i, _vp, _sz, _i, _c.POINTER(_u32)]),
    "alv_ffn_weight_create": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _i, _i, _i, _c.POINTER(_u32)]),
    "alv_weight_destroy": (_i, [_vp, _u32]),
    "alv_ffn_set_activation": (_i, [_vp, _u32, _i]),
    "alv_weight_info": (_i, [_vp, _u32, _c.POINTER(_c.c_int64)]),
    "alv_weight_dequantize": (_i, [_vp, _u32, _i, _vp, _vp]),
    "alv_gemv": (_i, [_vp, _u32, _i, _vp, _i, _vp, _i, _vp]),
    "alv_ffn": (_i, [_vp, _u32, _i, _vp, _i, _vp, _i, _vp]),
    "alv_ffn_layer": (_i, [_vp, _u32, _i, _vp, _vp, _vp, _vp, _vp]),
    "alv_ffn_stack_finalize": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp]),
    "alv_ffn_stack_create": (_i, [_vp, _c.POINTER(_u32), _i, _c.POINTER(_u32)]),
    "alv_ffn_stack_run": (_i, [_vp, _u32, _i, _vp, _vp, _vp]),
    "alv_activation": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp]),
    "alv_ffn_stack_exchange": (_i, [_vp, _u32, _i, _vp]),
    "alv_ffn_stack_connect": (_i, [_vp, _u32, _i, _i, _vp]),
    "alv_run_gemv": (_i, [_vp, _u32, _i, _vp, _i, _vp, _i]),
    "alv_run_ffn": (_i, [_vp, _u32, _i, _vp, _i, _vp, _i]),
    "alv_gemv_noalloc": (_i, [_vp, _u32, _i, _vp, _i, _vp, _i, _vp]),
    "alv_gemm": (_i, [_vp, _u32, _i, _vp, _vp, _i, _vp]),
    "alv_set_trace": (_i, [_vp, _vp]),
    "alv_ctx_info": (_i, [_vp, _c.POINTER(_c.c_int64)]),
    "alv_ffn_stack_set_probe": (_i, [_vp, _u32, _vp]),
    "alv_llama_create": (_i, [_vp, _vp, _c.POINTER(_u32)]),
    "alv_llama_load": (_i, [_vp, _u32, _c.c_char_p, _vp, _sz, _i]),
    "alv_llama_start": (_i, [_vp, _u32, _vp, _i, _vp]),
    "alv_llama_run": (_i, [_vp, _u32, _i, _i, _vp]),
    "alv_llama_tokens": (_i, [_vp, _u32, _i, _i, _vp, _vp]),
    "alv_llama_predicted": (_i, [_vp, _u32, _i, _i, _vp, _vp]),
    "alv_llama_generate": (_i, [_vp, _u32, _vp, _i, _i, _vp, _vp]),
    "alv_llama_forward": (_i, [_vp, _u32, _i, _i, _vp, _vp]),
    "alv_llama_reset": (_i, [_vp, _u32, _vp]),
    "alv_llama_info": (_i, [_vp, _u32, _vp]),
    "alv_llama_prefill": (_i, [_vp, _u32, _i, _i, _vp]),
}

_lock = threading.Lock()
_lib = None


class AlvError(RuntimeError):
    """A non-zero alv_status from the native library."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


def load() -> ctypes.CDLL:
    """Load the native library (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"alveare_b200 native library missing at {LIB_PATH}; "
                    "build it with `python -m alveare_b200.build`")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
        return _lib


class Context:
    """One alv_ctx on one CUDA device (NpuRegistry's lifetime, npu.h:48-51)."""

    def __init__(self, device: int = 0):
        self.lib = load()
        self.device = device
        p = _vp()
        rc = self.lib.alv_ctx_create(device, _c.byref(p))
        if rc:
            raise AlvError(rc, f"alv_ctx_create(device={device}) failed")
        self.ptr = p

    def check(self, rc: int, what: str) -> None:
        if rc:
            msg = self.lib.alv_last_error(self.ptr)
            raise AlvError(rc, f"{what}: {msg.decode() if msg else ''}")

    def sync_status(self, stream: int | None = None) -> None:
        self.check(self.lib.alv_sync_status(self.ptr, stream), "alv_sync_status")

    def info(self) -> dict:
        """alv_ctx_info as a dict."""
        out = (_c.c_int64 * 8)()
        self.check(self.lib.alv_ctx_info(self.ptr, out), "alv_ctx_info")
        keys = ("device", "num_sms", "scratch_bytes", "io_bytes", "allocs", "handles")
        return dict(zip(keys, list(out)[:6]))

    def close(self) -> None:
        if self.ptr:
            self.lib.alv_ctx_destroy(self.ptr)
            self.ptr = None


_contexts: dict[int, Context] = {}


def context(device: int = 0) -> Context:
    """Process-wide context for `device` (created on first use)."""
    with _lock:
        ctx = _contexts.get(device)
    if ctx is None:
        ctx = Context(device)
        with _lock:
            _contexts[device] = ctx
    return ctx
