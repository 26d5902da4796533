"""Reference-compatible Q4 operators on the B200.

Same names, keyword-only shape arguments and in-place outputs as the
reference's NPU operators, so ``runtime/py`` can switch by import:

* ``gemv_q_npu(W_combined, X, Y, *, N, K, m, k_tile)``  -- kernels/gemv_q/gemv_q.py:33-43
* ``ffn_fused_npu(W_fused, X, Y_partial, *, H, I, m_I, k_tile, activation)``
  -- kernels/ffn_fused/ffn_fused.py:28-39
* ``gemm_q_npu(W_combined, X, Y, *, B, N, K, m, k_tile)`` -- kernels/gemm_q/gemm_q.py:28-39
* ``pack_ffn_fused_weights(w_gate, w_up, w_down, H, I, m_I, k_tile)``
  -- kernels/ffn_fused/ffn_fused.py:330-395

Tensors are torch CUDA tensors (stream-ordered on the current stream) or host
numpy arrays (synchronous copy in / copy out, like the reference's
``_sync_to_device``).  ``m``, ``k_tile`` and ``m_I`` are NPU tiling knobs;
they are accepted and ignored.  A raw ``W_combined`` buffer is repacked into
the GPU layout on its first use and the resident copy is reused while the
same buffer (same object, address and size; for a torch tensor the same
version counter, for a host array the same fingerprint of 4 KB sampled over
it) comes back, the way the reference keeps its weights resident
(model.py:41-53); :class:`Q4Weight` registers one explicitly, and
:func:`clear_weight_cache` drops the cached copies (call it after changing a
few bytes of a host array, or a tensor by other means than torch).
"""
from __future__ import annotations

import ctypes
import zlib
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import ACT_GELU, ACT_SILU, BF16, F32, context

try:  # torch is plumbing (device memory, streams); numpy host arrays also work
    import torch
except Exception:  # pragma: no cover
    torch = None

_ACT = {"gelu": ACT_GELU, "silu": ACT_SILU}


# ---------------------------------------------------------------------------
# buffer helpers
# ---------------------------------------------------------------------------
def _is_torch(t) -> bool:
    return torch is not None and isinstance(t, torch.Tensor)


def _dtype_code(t) -> int:
    if _is_torch(t):
        if t.dtype == torch.float32:
            return F32
        if t.dtype == torch.bfloat16:
            return BF16
        raise TypeError(f"unsupported activation dtype {t.dtype} (float32 or bfloat16)")
    name = np.asarray(t).dtype.name
    if name == "float32":
        return F32
    if name == "bfloat16":
        return BF16
    raise TypeError(f"unsupported activation dtype {name} (float32 or bfloat16)")


def _device_of(*ts) -> int | None:
    for t in ts:
        if _is_torch(t) and t.is_cuda:
            return t.device.index if t.device.index is not None else torch.cuda.current_device()
    return None


def _stream(device: int) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _cuda_ptr(t) -> int:
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return t.data_ptr()


def _host_array(a) -> np.ndarray:
    if _is_torch(a):
        a = a.detach().cpu()
        if a.dtype == torch.bfloat16:
            from ml_dtypes import bfloat16
            return np.ascontiguousarray(a.view(torch.int16).numpy().view(bfloat16))
        return np.ascontiguousarray(a.numpy())
    return np.ascontiguousarray(a)


# ---------------------------------------------------------------------------
# registered weights
# ---------------------------------------------------------------------------
class Q4Weight:
    """An (N, K) Q4 matrix resident on a GPU in the library's unit layout.

    Built from the reference's packed (N, K/32*20) uint8 layout (host numpy or
    torch, CPU or CUDA).  ``shape`` mirrors the packed array's shape so code
    that derives N and K from ``W.shape`` keeps working (model.py:284-293).
    """

    def __init__(self, W_combined, N: int | None = None, K: int | None = None, device: int | None = None):
        dev = _device_of(W_combined)
        device = dev if device is None else device
        device = 0 if device is None else device
        self.ctx = context(device)
        self.device = device
        if N is None:
            N = int(W_combined.shape[0])
        if K is None:
            K = int(W_combined.shape[-1]) // 20 * 32 if len(W_combined.shape) == 2 else None
        if K is None:
            raise ValueError("K is required for a flat W_combined")
        self.N, self.K = int(N), int(K)
        nbytes = self.N * (self.K // 32) * 20
        h = ctypes.c_uint32()
        if _is_torch(W_combined) and W_combined.is_cuda:
            if W_combined.numel() * W_combined.element_size() != nbytes:
                raise ValueError(f"W_combined has {W_combined.numel()} bytes, expected {nbytes}")
            torch.cuda.current_stream(device).synchronize()
            rc = self.ctx.lib.alv_gemv_weight_create(self.ctx.ptr, self.N, self.K, _cuda_ptr(W_combined),
                                                     nbytes, 1, ctypes.byref(h))
        else:
            arr = np.ascontiguousarray(_host_array(W_combined), dtype=np.uint8)
            if arr.size != nbytes:
                raise ValueError(f"W_combined has {arr.size} bytes, expected {nbytes}")
            rc = self.ctx.lib.alv_gemv_weight_create(self.ctx.ptr, self.N, self.K, arr.ctypes.data,
                                                     nbytes, 0, ctypes.byref(h))
        self.ctx.check(rc, "alv_gemv_weight_create")
        self.handle = h.value
        self.shape = (self.N, (self.K // 32) * 20)

    def info(self) -> list[int]:
        out = (ctypes.c_int64 * 8)()
        self.ctx.check(self.ctx.lib.alv_weight_info(self.ctx.ptr, self.handle, out), "alv_weight_info")
        return list(out)

    def dequantize(self):
        """bf16 (N, K) torch tensor on the GPU (dequantize_combined on device)."""
        out = torch.empty((self.N, self.K), dtype=torch.bfloat16, device=f"cuda:{self.device}")
        self.ctx.check(self.ctx.lib.alv_weight_dequantize(self.ctx.ptr, self.handle, 0, out.data_ptr(),
                                                          _stream(self.device)), "alv_weight_dequantize")
        return out

    def free(self) -> None:
        if self.handle:
            self.ctx.lib.alv_weight_destroy(self.ctx.ptr, self.handle)
            self.handle = 0


class FusedFFNWeight:
    """gate/up/down of one FFN (optionally an intermediate-dim slice for
    tensor parallelism) resident on a GPU.  Stands in for the reference's
    ``W_fused`` per-core tile stream; ``n_cores`` is 1, so ``Y_partial`` has
    one row and the reference's host partial sum is the identity
    (model.py:394-395, npu.cpp:360-377)."""

    n_cores = 1

    def __init__(self, w_gate, w_up, w_down, H: int, I: int, activation: str = "gelu",
                 device: int | None = None, i_begin: int = 0, i_end: int | None = None):
        dev = _device_of(w_gate, w_up, w_down)
        device = dev if device is None else device
        device = 0 if device is None else device
        self.ctx = context(device)
        self.device = device
        self.H, self.I = int(H), int(I)
        self.i_begin = int(i_begin)
        self.i_end = self.I if i_end is None else int(i_end)
        self.activation = activation
        gb = self.I * (self.H // 32) * 20
        db = self.H * (self.I // 32) * 20
        h = ctypes.c_uint32()
        on_dev = all(_is_torch(w) and w.is_cuda for w in (w_gate, w_up, w_down))
        if on_dev:
            for w, n in ((w_gate, gb), (w_up, gb), (w_down, db)):
                if w.numel() * w.element_size() != n:
                    raise ValueError("FFN weight buffer has the wrong size")
            torch.cuda.current_stream(device).synchronize()
            ptrs = [_cuda_ptr(w) for w in (w_gate, w_up, w_down)]
        else:
            keep = [np.ascontiguousarray(_host_array(w), dtype=np.uint8) for w in (w_gate, w_up, w_down)]
            for a, n in zip(keep, (gb, gb, db)):
                if a.size != n:
                    raise ValueError("FFN weight buffer has the wrong size")
            ptrs = [a.ctypes.data for a in keep]
        rc = self.ctx.lib.alv_ffn_weight_create(self.ctx.ptr, self.H, self.I, _ACT[activation], *ptrs,
                                                1 if on_dev else 0, self.i_begin, self.i_end, ctypes.byref(h))
        self.ctx.check(rc, "alv_ffn_weight_create")
        self.handle = h.value
        self.shape = (1, (2 * (self.i_end - self.i_begin) * (self.H // 32) + self.H * ((self.i_end - self.i_begin) // 32)) * 20)

    def set_activation(self, activation: str) -> None:
        if activation != self.activation:
            self.ctx.check(self.ctx.lib.alv_ffn_set_activation(self.ctx.ptr, self.handle, _ACT[activation]),
                           "alv_ffn_set_activation")
            self.activation = activation

    def info(self) -> list[int]:
        out = (ctypes.c_int64 * 8)()
        self.ctx.check(self.ctx.lib.alv_weight_info(self.ctx.ptr, self.handle, out), "alv_weight_info")
        return list(out)

    def dequantize(self, which: int):
        rows = self.H if which == 2 else self.i_end - self.i_begin
        cols = self.i_end - self.i_begin if which == 2 else self.H
        out = torch.empty((rows, cols), dtype=torch.bfloat16, device=f"cuda:{self.device}")
        self.ctx.check(self.ctx.lib.alv_weight_dequantize(self.ctx.ptr, self.handle, which, out.data_ptr(),
                                                          _stream(self.device)), "alv_weight_dequantize")
        return out

    def free(self) -> None:
        if self.handle:
            self.ctx.lib.alv_weight_destroy(self.ctx.ptr, self.handle)
            self.handle = 0


# ---------------------------------------------------------------------------
# generic launch helpers
# ---------------------------------------------------------------------------
def _run(ctx, kind: str, handle: int, ntok: int, X, Y, device: int) -> None:
    lib = ctx.lib
    xd, yd = _dtype_code(X), _dtype_code(Y)
    if _is_torch(X) and X.is_cuda:
        if not (_is_torch(Y) and Y.is_cuda):
            raise ValueError("X on the GPU needs Y on the GPU")
        fn = lib.alv_gemv if kind == "gemv" else lib.alv_ffn
        ctx.check(fn(ctx.ptr, handle, ntok, _cuda_ptr(X), xd, _cuda_ptr(Y), yd, _stream(device)), f"alv_{kind}")
        return
    # host buffers: synchronous copy in / run / copy out
    xa = _host_array(X)
    if _is_torch(Y):
        if Y.is_cuda:
            raise ValueError("host X needs a host Y")
        ya = np.empty(tuple(Y.shape), dtype=np.float32 if yd == F32 else _host_array(Y).dtype)
    else:
        ya = Y
        if not ya.flags["C_CONTIGUOUS"]:
            raise ValueError("Y must be contiguous")
    fn = lib.alv_run_gemv if kind == "gemv" else lib.alv_run_ffn
    ctx.check(fn(ctx.ptr, handle, ntok, xa.ctypes.data, xd, ya.ctypes.data, yd), f"alv_run_{kind}")
    if _is_torch(Y):
        if yd == F32:
            Y.copy_(torch.from_numpy(ya))
        else:
            Y.copy_(torch.from_numpy(ya.view(np.int16)).view(torch.bfloat16))


# Raw packed buffers seen by the operators -> their resident Q4Weight.  The
# source object is held, so its address cannot be reused by another buffer
# while the entry lives.
_WEIGHT_CACHE: dict = {}


def _buffer_key(W, N: int, K: int, device):
    if _is_torch(W):
        dev = W.device.index if W.is_cuda else -1
        return ("torch", dev, W.data_ptr(), W.numel() * W.element_size(), N, K, device), W._version
    a = np.asarray(W)
    return ("host", -1, a.__array_interface__["data"][0], a.nbytes, N, K, device), _host_fingerprint(a)


def _host_fingerprint(a: np.ndarray) -> int:
    """crc32 of 64 windows of 64 bytes spread evenly over a host buffer (all
    of it up to 4 KB): a staging buffer refilled with another matrix gets a
    new fingerprint, so it is repacked again, without reading it whole."""
    b = np.ascontiguousarray(a).reshape(-1).view(np.uint8)
    if b.size <= 4096:
        return zlib.crc32(b.tobytes())
    starts = np.linspace(0, b.size - 64, 64).astype(np.int64)
    return zlib.crc32(b[(starts[:, None] + np.arange(64)).reshape(-1)].tobytes())


def clear_weight_cache() -> None:
    """Free every resident copy made for a raw W_combined buffer."""
    for _, _, w in list(_WEIGHT_CACHE.values()):
        w.free()
    _WEIGHT_CACHE.clear()


def _as_weight(W, N, K, device):
    if isinstance(W, Q4Weight):
        if W.N != N or W.K != K:
            raise ValueError(f"weight is ({W.N}, {W.K}), call asked for ({N}, {K})")
        return W
    key, version = _buffer_key(W, N, K, device)
    hit = _WEIGHT_CACHE.get(key)
    if hit is not None and hit[0] is W and hit[1] == version:
        return hit[2]
    if hit is not None:
        hit[2].free()
    w = Q4Weight(W, N=N, K=K, device=device)
    _WEIGHT_CACHE[key] = (W, version, w)
    return w


# ---------------------------------------------------------------------------
# reference operator signatures
# ---------------------------------------------------------------------------
def gemv_q_npu(W_combined, X, Y, *, N: int, K: int, m: int = 32, k_tile: int = 256) -> None:
    """Y[N] = W[N, K] @ X[K] for the Q4 matrix W (kernels/gemv_q/gemv_q.py:33-43).
    Y is written in place (fp32 or bf16)."""
    device = _device_of(X, Y, W_combined)
    w = _as_weight(W_combined, N, K, device)
    if int(np.prod(X.shape)) < K or int(np.prod(Y.shape)) < N:
        raise ValueError("X or Y too small for (N, K)")
    Xv = X[:K] if X.shape[0] > K and len(X.shape) == 1 else X
    Yv = Y[:N] if Y.shape[0] > N and len(Y.shape) == 1 else Y
    _run(w.ctx, "gemv", w.handle, 1, Xv, Yv, w.device)


# Batches above this many bf16 tokens run on the tcgen05 prefill kernel; the
# decode-sized ones stay on the HBM-bound streaming gemv.
GEMM_TC_MIN_TOKENS = 17


def _gemm_tc(w, B: int, Xv, Yv) -> None:
    """Y = X W^T through alv_gemm (bf16 X on the device, 16-byte aligned)."""
    ctx, device = w.ctx, w.device
    yd = _dtype_code(Yv)
    if _is_torch(Xv) and Xv.is_cuda:
        xt = Xv.contiguous()
    else:
        xt = torch.from_numpy(np.ascontiguousarray(_host_array(Xv)).view(np.int16)).to(
            torch.device("cuda", device)).view(torch.bfloat16)
    if xt.data_ptr() % 16:
        xt = xt.clone()
    on_dev = _is_torch(Yv) and Yv.is_cuda
    if on_dev and Yv.is_contiguous():
        yt = Yv
    else:
        yt = torch.empty((B, Yv.shape[-1]), dtype=torch.float32 if yd == F32 else torch.bfloat16,
                         device=torch.device("cuda", device))
    ctx.check(ctx.lib.alv_gemm(ctx.ptr, w.handle, B, xt.data_ptr(), yt.data_ptr(), yd, _stream(device)), "alv_gemm")
    if yt is not Yv:
        if on_dev:
            Yv.copy_(yt)
        else:
            torch.cuda.current_stream(device).synchronize()
            ctx.sync_status(_stream(device))
            host = yt.cpu()
            if _is_torch(Yv):
                Yv.copy_(host)
            elif yd == F32:
                Yv[...] = host.numpy()
            else:
                Yv[...] = host.view(torch.int16).numpy().view(Yv.dtype)


def gemm_q_npu(W_combined, X, Y, *, B: int, N: int, K: int, m: int = 32, k_tile: int = 256) -> None:
    """Y[B, N] = X[B, K] @ W^T for the Q4 matrix W (kernels/gemm_q/gemm_q.py:28-39).
    bf16 batches of GEMM_TC_MIN_TOKENS or more run on the tensor cores
    (tcgen05); smaller ones (and fp32 X) are processed by the streaming gemv
    in slices of 16 (8 for fp32) tokens."""
    device = _device_of(X, Y, W_combined)
    w = _as_weight(W_combined, N, K, device)
    Xv = X.reshape(B, K) if not (len(X.shape) == 2 and tuple(X.shape) == (B, K)) else X
    Yv = Y.reshape(B, N) if not (len(Y.shape) == 2 and tuple(Y.shape) == (B, N)) else Y
    if _dtype_code(X) == BF16 and B >= GEMM_TC_MIN_TOKENS:
        _gemm_tc(w, B, Xv, Yv)
        return
    step = 16 if _dtype_code(X) == BF16 else 8
    for b0 in range(0, B, step):
        b1 = min(B, b0 + step)
        xs, ys = Xv[b0:b1], Yv[b0:b1]
        if _is_torch(ys) or not ys.flags["C_CONTIGUOUS"]:
            _run(w.ctx, "gemv", w.handle, b1 - b0, xs, ys, w.device)
        else:
            _run(w.ctx, "gemv", w.handle, b1 - b0, np.ascontiguousarray(xs), ys, w.device)


def pack_ffn_fused_weights(w_gate, w_up, w_down, H: int, I: int, m_I: int = 32, k_tile: int = 256,
                           activation: str = "gelu", device: int | None = None) -> FusedFFNWeight:
    """Load-time FFN repack (kernels/ffn_fused/ffn_fused.py:330-395): takes the
    three packed (rows, cols/32*20) matrices and returns the resident fused
    weight consumed by :func:`ffn_fused_npu`."""
    return FusedFFNWeight(w_gate, w_up, w_down, H, I, activation=activation, device=device)


def ffn_fused_npu(W_fused, X, Y_partial, *, H: int, I: int, m_I: int = 32, k_tile: int = 256,
                  activation: str = "gelu") -> None:
    """Fused FFN (kernels/ffn_fused/ffn_fused.py:28-39).  Writes the full
    y = Wd act(Wg x, Wu x) into row 0 of Y_partial and zeros the other rows,
    so summing Y_partial over its first axis (the reference host reduction)
    returns y.

    X may also hold a batch of 1..8 tokens, (B, H); Y_partial is then
    (n_rows, B, H) with y in row 0, or (B, H)."""
    if not isinstance(W_fused, FusedFFNWeight):
        raise TypeError("W_fused must come from alveare_b200.pack_ffn_fused_weights")
    if W_fused.H != H or W_fused.I != I:
        raise ValueError(f"W_fused is (H={W_fused.H}, I={W_fused.I}), call asked for ({H}, {I})")
    W_fused.set_activation(activation)
    if len(X.shape) == 2 and X.shape[0] > 1:
        ntok = int(X.shape[0])
        if not 1 <= ntok <= 8:
            raise ValueError("ffn_fused_npu: a batch holds 1..8 tokens")
        if tuple(Y_partial.shape[-2:]) != (ntok, H):
            raise ValueError(f"Y_partial must end in ({ntok}, {H})")
        if len(Y_partial.shape) == 3:
            if Y_partial.shape[0] > 1:
                Y_partial[1:] = 0
            y0 = Y_partial[0]
        else:
            y0 = Y_partial
        _run(W_fused.ctx, "ffn", W_fused.handle, ntok, X, y0, W_fused.device)
        return
    Yp = Y_partial.reshape(-1, H) if Y_partial.shape[-1] != H or len(Y_partial.shape) != 2 else Y_partial
    if Yp.shape[0] > 1:
        Yp[1:] = 0
    y0 = Yp[0]
    Xv = X.reshape(-1)[:H] if len(X.shape) == 2 else (X[:H] if X.shape[0] > H else X)
    _run(W_fused.ctx, "ffn", W_fused.handle, 1, Xv, y0, W_fused.device)


def q4_quantize(W):
    """GPU quantize_to_q4_0 + pack_to_combined (tools/convert/gemv_q_convert.py:5-85)
    of a float32 (N, K) CUDA tensor; returns the (N, K/32*20) uint8 CUDA tensor."""
    if not (_is_torch(W) and W.is_cuda and W.dtype == torch.float32 and W.dim() == 2):
        raise TypeError("W must be a 2-D float32 CUDA tensor")
    N, K = W.shape
    device = W.device.index
    ctx = context(device)
    out = torch.empty((N, K // 32 * 20), dtype=torch.uint8, device=W.device)
    ctx.check(ctx.lib.alv_q4_quantize(ctx.ptr, _cuda_ptr(W), N, K, out.data_ptr(), _stream(device)),
              "alv_q4_quantize")
    return out
