"""alv_gemv_noalloc: the gemv entry point for callers that may not allocate
device memory while they run (fixed GPU memory budget, an allocator owned by
the host runtime, no tolerance for the synchronization of cudaMalloc).  It
keeps its split-K workspace in a static device array instead of the
context's growable scratch arena.

Checked against alv_gemv, through the C ABI, on two calls in a row (the
static array keeps the previous call's contents, so the second call shows the
counters were cleared), within the 1e-4 normwise tolerance of the gemv tests.
Collected last so a failure here does not stop the rest of a -x run."""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from alveare_b200 import Q4Weight, _lib  # noqa: E402
from oracle import q4  # noqa: E402

TIGHT = 1e-4


def normwise(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def _call(fn, w, ntok, x, y):
    ctx = w.ctx
    rc = fn(ctx.ptr, w.handle, ntok, x.data_ptr(), _lib.F32 if x.dtype == torch.float32 else _lib.BF16,
            y.data_ptr(), _lib.F32, torch.cuda.current_stream().cuda_stream)
    ctx.check(rc, fn.__name__)
    ctx.sync_status()
    return y.cpu().numpy().copy()


@pytest.mark.parametrize("N,K,ntok", [(3840, 15360, 1), (6912, 1152, 1), (1152, 6912, 2)])
def test_noalloc_gemv_matches_gemv_twice(N, K, ntok):
    rng = np.random.default_rng(N + K + ntok)
    comb = q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    w = Q4Weight(comb)
    lib = w.ctx.lib
    x = torch.from_numpy(rng.normal(0, 1, (ntok, K)).astype(np.float32)).cuda()
    y = torch.empty((ntok, N), dtype=torch.float32, device="cuda")
    ref = _call(lib.alv_gemv, w, ntok, x, y)
    for _ in range(2):
        y.fill_(float("nan"))
        got = _call(lib.alv_gemv_noalloc, w, ntok, x, y)
        assert normwise(got, ref) <= TIGHT
    assert normwise(ref, q4.gemv_q(comb, x.cpu().numpy())) <= TIGHT
    w.free()


def test_noalloc_gemv_rejects_sizes_beyond_its_static_array():
    rng = np.random.default_rng(9)
    comb = q4.quantize_combined(rng.normal(0, 0.02, (64, 256)).astype(np.float32))
    w = Q4Weight(comb)
    x = torch.zeros((5, 256), dtype=torch.bfloat16, device="cuda")
    y = torch.empty((5, 64), dtype=torch.float32, device="cuda")
    rc = w.ctx.lib.alv_gemv_noalloc(w.ctx.ptr, w.handle, 5, x.data_ptr(), _lib.BF16, y.data_ptr(), _lib.F32,
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 6  # ALV_ERR_UNSUPPORTED
    assert b"ntok" in w.ctx.lib.alv_last_error(w.ctx.ptr)
    w.free()
