"""alv_gemv_noalloc: the gemv entry point for callers that may not allocate
device memory while they run -- a decode loop whose GPU memory budget is
fixed at start-up, a host runtime that owns the device allocator, or code
that cannot afford the device synchronization a cudaMalloc/cudaFree brings.
It keeps its split-K workspace in a static device array instead of the
context's growable scratch arena.

Checked through the C ABI: on a context of its own, before any other gemv
ran on it, the entry point makes no device allocation (the context's
allocation count is unchanged), and its output matches alv_gemv within the
1e-4 normwise tolerance of the gemv tests on two calls in a row (the static
array keeps the previous call's contents, so the second call shows the
counters were cleared).  fp32 and bf16 activations.  Collected last so a
failure here does not stop the rest of a -x run."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from alveare_b200 import _lib  # noqa: E402
from oracle import q4  # noqa: E402

TIGHT = 1e-4


def normwise(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _dtype(t):
    return _lib.F32 if t.dtype == torch.float32 else _lib.BF16


def _call(ctx, fn, handle, ntok, x, y):
    rc = fn(ctx.ptr, handle, ntok, x.data_ptr(), _dtype(x), y.data_ptr(), _dtype(y),
            torch.cuda.current_stream().cuda_stream)
    ctx.check(rc, fn.__name__)
    ctx.sync_status()
    return y.float().cpu().numpy().copy()


@pytest.mark.parametrize("N,K,ntok,xdt,ydt", [
    (3840, 15360, 1, torch.float32, torch.float32),
    (6912, 1152, 1, torch.float32, torch.float32),
    (1152, 6912, 2, torch.float32, torch.float32),
    (2048, 2048, 4, torch.bfloat16, torch.bfloat16),
])
def test_noalloc_gemv_matches_gemv_twice(N, K, ntok, xdt, ydt):
    rng = np.random.default_rng(N + K + ntok)
    comb = q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    ctx = _lib.Context(0)          # a context of its own: nothing has run on it yet
    try:
        import ctypes
        h = ctypes.c_uint32()
        ctx.check(ctx.lib.alv_gemv_weight_create(ctx.ptr, N, K, comb.ctypes.data, comb.nbytes, 0,
                                                 ctypes.byref(h)), "alv_gemv_weight_create")
        x = torch.from_numpy(rng.normal(0, 1, (ntok, K)).astype(np.float32)).cuda().to(xdt)
        y = torch.empty((ntok, N), dtype=ydt, device="cuda")
        allocs = ctx.info()["allocs"]
        outs = []
        for _ in range(2):
            y.fill_(float("nan"))
            outs.append(_call(ctx, ctx.lib.alv_gemv_noalloc, h.value, ntok, x, y))
        assert ctx.info()["allocs"] == allocs      # no device allocation by the no-alloc calls
        ref = _call(ctx, ctx.lib.alv_gemv, h.value, ntok, x, y)
        for got in outs:
            if ydt == torch.float32:
                assert normwise(got, ref) <= TIGHT
            else:                                   # same fp32 sums, same bf16 rounding
                assert np.array_equal(got, ref)
        assert normwise(ref, q4.gemv_q(comb, x.float().cpu().numpy())) <= (TIGHT if ydt == torch.float32 else 1e-2)
        ctx.check(ctx.lib.alv_weight_destroy(ctx.ptr, h.value), "alv_weight_destroy")
    finally:
        ctx.close()


def test_noalloc_gemv_rejects_sizes_beyond_its_static_array():
    import ctypes
    rng = np.random.default_rng(9)
    comb = q4.quantize_combined(rng.normal(0, 0.02, (64, 256)).astype(np.float32))
    ctx = _lib.context(0)
    h = ctypes.c_uint32()
    ctx.check(ctx.lib.alv_gemv_weight_create(ctx.ptr, 64, 256, comb.ctypes.data, comb.nbytes, 0, ctypes.byref(h)),
              "alv_gemv_weight_create")
    x = torch.zeros((5, 256), dtype=torch.bfloat16, device="cuda")
    y = torch.empty((5, 64), dtype=torch.float32, device="cuda")
    rc = ctx.lib.alv_gemv_noalloc(ctx.ptr, h.value, 5, x.data_ptr(), _lib.BF16, y.data_ptr(), _lib.F32,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 6  # ALV_ERR_UNSUPPORTED
    assert b"ntok" in ctx.lib.alv_last_error(ctx.ptr)
    ctx.check(ctx.lib.alv_weight_destroy(ctx.ptr, h.value), "alv_weight_destroy")
