"""gemv_q on the B200 vs the CPU oracle (oracle/q4.py, pinned to the
reference).  Tolerance (north star): max|y - y_ref| / max|y_ref| <= 1e-3 on
fp32 outputs; the kernels accumulate exact bf16 products in fp32, so the
tests also assert a 1e-4 bound to catch silent arithmetic drift.
Integer/byte work (quantize, repack, dequantize) must be bit-exact."""
import hashlib
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from alveare_b200 import Q4Weight, _lib, gemm_q_npu, gemv_q_npu, q4_quantize  # noqa: E402
from oracle import q4  # noqa: E402

TOL = 1e-3
TIGHT = 1e-4


def normwise(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def run_gemv(w, x, ntok=1, out_dtype=torch.float32):
    xt = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    if xt.dtype == torch.int16:
        xt = xt.view(torch.bfloat16)
    y = torch.empty((ntok, w.N) if ntok > 1 else (w.N,), dtype=out_dtype, device="cuda")
    if ntok == 1:
        gemv_q_npu(w, xt, y, N=w.N, K=w.K)
    else:
        gemm_q_npu(w, xt, y, B=ntok, N=w.N, K=w.K)
    w.ctx.sync_status()
    return y.float().cpu().numpy()


def bf16_np(a):
    """float32 -> bf16 bits as int16 numpy (torch-friendly)."""
    return q4.bf16_bits(a).view(np.int16)


# ---------------------------------------------------------------- quantizer
def test_gpu_quantizer_matches_reference_golden(golden_dir):
    g = np.load(os.path.join(golden_dir, "quant_64x256.npz"))
    out = q4_quantize(torch.from_numpy(g["W"]).cuda()).cpu().numpy()
    np.testing.assert_array_equal(out, g["combined"])


def test_gpu_quantizer_config1_hash(golden_dir):
    h = json.loads(open(os.path.join(golden_dir, "hashes.json")).read())
    rng = np.random.default_rng(0)
    W = rng.normal(0, 0.02, (6912, 1152)).astype(np.float32)
    out = q4_quantize(torch.from_numpy(W).cuda()).cpu().numpy()
    assert hashlib.sha256(out.tobytes()).hexdigest() == h["config1_combined"]


# ---------------------------------------------------------------- dequant
def _scale_matrix(scale_bits, rng):
    """One 32-block per scale; the nibbles of each block cover all 16 codes twice."""
    n = len(scale_bits)
    kb = 32
    rows = (n + kb - 1) // kb
    sb = np.zeros(rows * kb, np.uint16)
    sb[:n] = scale_bits
    sb = sb.reshape(rows, kb)
    codes = np.arange(16, dtype=np.uint8)
    nib = np.empty((rows, kb, 16), np.uint8)
    for r in range(rows):
        for b in range(kb):
            p = rng.permutation(16).astype(np.uint8)
            lo = codes[p]
            hi = codes[np.roll(p, 5)]
            nib[r, b] = (lo & 15) | ((hi & 15) << 4)
    return q4.pack_to_combined(nib.reshape(rows, kb * 16), sb)


def _check_dequant(comb):
    """Bit-exact except that a zero product may carry either sign (q = 0 with a
    negative scale gives -0 in numpy and +0 on the fast path; equal as numbers)."""
    w = Q4Weight(comb)
    got = w.dequantize().view(torch.int16).cpu().numpy().view(np.uint16)
    ref = q4.bf16_bits(q4.dequantize_combined(comb))
    nan_ref = np.isnan(q4.bits_to_f32(ref))
    nan_got = np.isnan(q4.bits_to_f32(got))
    np.testing.assert_array_equal(nan_got, nan_ref)
    zero = (ref & 0x7FFF) == 0
    np.testing.assert_array_equal(got[~nan_ref & ~zero], ref[~nan_ref & ~zero])
    assert np.all((got[zero] & 0x7FFF) == 0)
    return w


def test_dequant_fast_path_bit_exact_over_scale_range():
    rng = np.random.default_rng(1)
    # every bf16 scale with exponent in [-40, 4], both signs: inside the fast window
    bits = [(s << 15) | (e << 7) | m for s in (0, 1) for e in range(127 - 40, 127 + 5) for m in range(128)]
    w = _check_dequant(_scale_matrix(np.array(bits, np.uint16), rng))
    assert w.info()[3] == 1, "expected the fast dequant path"


def test_dequant_generic_path_bit_exact_all_scales():
    rng = np.random.default_rng(2)
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)  # every pattern incl. inf/nan/subnormal
    w = _check_dequant(_scale_matrix(bits, rng))
    assert w.info()[3] == 0, "expected the generic dequant path"


def test_dequant_wide_but_finite_range_uses_generic():
    rng = np.random.default_rng(3)
    bits = np.array([0x0100, 0x4000, 0x3F80, 0x3C00], np.uint16)  # 2^-125 .. 2
    w = _check_dequant(_scale_matrix(bits, rng))
    assert w.info()[3] == 0


# ---------------------------------------------------------------- gemv parity
def test_gemv_random_bytes_golden(golden_dir):
    g = np.load(os.path.join(golden_dir, "randbytes_48x256.npz"))
    w = Q4Weight(g["combined"])
    y = run_gemv(w, g["x"])
    e = normwise(y, g["y32"])
    assert e <= TOL and e <= TIGHT, e


def test_gemv_reference_unit_test_case(golden_dir):
    """tests/test_gemv_q.py:76-94 of the reference: bf16 x, 256x256."""
    g = np.load(os.path.join(golden_dir, "ref_test_tiny_256.npz"))
    w = Q4Weight(torch.from_numpy(g["combined"]).cuda())
    y = run_gemv(w, bf16_np(g["x"]))
    e = normwise(y, g["y32"])
    assert e <= TIGHT, e
    # bf16 output path
    yb = run_gemv(w, bf16_np(g["x"]), out_dtype=torch.bfloat16)
    assert np.mean(q4.bf16_bits(yb) == g["y_bf16_bits"]) > 0.97


def test_gemv_config1_fp32():
    rng = np.random.default_rng(0)
    W = rng.normal(0, 0.02, (6912, 1152)).astype(np.float32)
    x = rng.normal(0, 1, 1152).astype(np.float32)
    comb = q4.quantize_combined(W)
    w = Q4Weight(torch.from_numpy(comb).cuda())
    assert w.info()[3] == 1
    ref = q4.gemv_q(comb, x)
    y = run_gemv(w, x)
    e = normwise(y, ref)
    assert e <= TIGHT, e
    y2 = run_gemv(w, x)
    np.testing.assert_array_equal(y, y2)  # deterministic


@pytest.mark.parametrize("N,K", [(1, 32), (7, 96), (16, 64), (17, 160), (33, 32), (300, 1088),
                                 (2048, 2048), (1152, 6912), (257, 15360)])
def test_gemv_shapes(N, K):
    rng = np.random.default_rng(N * 7919 + K)
    comb = q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    x = rng.normal(0, 1, K).astype(np.float32)
    w = Q4Weight(comb)
    e = normwise(run_gemv(w, x), q4.gemv_q(comb, x))
    assert e <= TIGHT, (N, K, e)


@pytest.mark.parametrize("ntok", [1, 2, 3, 4, 5, 8, 9, 16])
def test_gemv_decode_batch_bf16(ntok):
    rng = np.random.default_rng(ntok)
    N, K = 640, 1024
    comb = q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    X = q4.to_bf16(rng.normal(0, 1, (ntok, K)).astype(np.float32))
    w = Q4Weight(comb)
    y = run_gemv(w, bf16_np(X), ntok=ntok)
    ref = q4.gemm_q(comb, X)
    assert normwise(y.reshape(ntok, N), ref.reshape(ntok, N)) <= TIGHT


@pytest.mark.parametrize("ntok", [2, 3, 8])
def test_gemv_decode_batch_fp32(ntok):
    rng = np.random.default_rng(100 + ntok)
    N, K = 512, 768
    comb = q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    X = rng.normal(0, 1, (ntok, K)).astype(np.float32)
    w = Q4Weight(comb)
    y = run_gemv(w, X, ntok=ntok)
    assert normwise(y, q4.gemm_q(comb, X)) <= TIGHT


def test_gemv_generic_path_parity():
    rng = np.random.default_rng(5)
    N, K = 96, 512
    comb = q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    v = comb.reshape(N, K // 32, 20)
    v[0, 0, 16:18] = [0x00, 0x01]   # a 2^-125 scale ...
    v[1, 0, 16:18] = [0x80, 0x40]   # ... and a 4.0 scale: 127 binades force the generic path
    w = Q4Weight(comb)
    assert w.info()[3] == 0
    x = rng.normal(0, 1, K).astype(np.float32)
    assert normwise(run_gemv(w, x), q4.gemv_q(comb, x)) <= TIGHT


def test_gemv_host_buffers_numpy():
    rng = np.random.default_rng(6)
    N, K = 384, 640
    comb = q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    x = rng.normal(0, 1, K).astype(np.float32)
    y = np.zeros(N, np.float32)
    gemv_q_npu(comb, x, y, N=N, K=K, m=32, k_tile=256)  # raw buffer, repacked per call
    assert normwise(y, q4.gemv_q(comb, x)) <= TIGHT


def test_gemv_zero_matrix_and_zero_x():
    N, K = 64, 128
    comb = q4.quantize_combined(np.zeros((N, K), np.float32))
    w = Q4Weight(comb)
    y = run_gemv(w, np.ones(K, np.float32))
    assert np.all(y == 0)


@pytest.mark.parametrize("xdt,off", [(torch.float32, 4), (torch.bfloat16, 2)])
def test_gemv_and_ffn_reject_misaligned_x_without_launching(xdt, off):
    """An activation view at an odd element offset (x[1:] of a buffer) is
    refused with ALV_ERR_ARG before any kernel is launched: the kernels read
    x in element pairs (8-byte fp32 / 4-byte bf16 loads)."""
    from alveare_b200 import FusedFFNWeight
    rng = np.random.default_rng(3)
    K, N = 256, 64
    w = Q4Weight(q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32)))
    buf = torch.zeros(K + 8, dtype=xdt, device="cuda")
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    code = _lib.F32 if xdt == torch.float32 else _lib.BF16
    st = torch.cuda.current_stream().cuda_stream
    ctx = w.ctx
    assert ctx.lib.alv_gemv(ctx.ptr, w.handle, 1, buf.data_ptr() + off, code, y.data_ptr(), _lib.F32, st) == 1
    assert b"aligned" in ctx.lib.alv_last_error(ctx.ptr)
    assert ctx.lib.alv_gemv_noalloc(ctx.ptr, w.handle, 1, buf.data_ptr() + off, code, y.data_ptr(), _lib.F32,
                                    st) == 1
    H, I = 256, 512
    f = FusedFFNWeight(*(q4.quantize_combined(rng.normal(0, 0.02, s).astype(np.float32))
                         for s in ((I, H), (I, H), (H, I))), H, I, "gelu")
    yf = torch.empty(H, dtype=torch.float32, device="cuda")
    assert ctx.lib.alv_ffn(ctx.ptr, f.handle, 1, buf.data_ptr() + off, code, yf.data_ptr(), _lib.F32, st) == 1
    ctx.sync_status()
    w.free()
    f.free()


def test_raw_buffer_is_repacked_once():
    """gemv_q_npu / gemm_q_npu given the reference's raw packed buffer repack
    it on the first call only: the second call with the same buffer reuses the
    resident copy (no new weight handle, no device allocation)."""
    from alveare_b200 import ops
    ops.clear_weight_cache()
    rng = np.random.default_rng(12)
    N, K = 512, 1024
    comb = torch.from_numpy(q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))).cuda()
    x = torch.from_numpy(rng.normal(0, 1, K).astype(np.float32)).cuda()
    y1 = torch.empty(N, device="cuda")
    y2 = torch.empty(N, device="cuda")
    ctx = _lib.context(0)
    gemv_q_npu(comb, x, y1, N=N, K=K)
    before = ctx.info()
    gemv_q_npu(comb, x, y2, N=N, K=K)
    X = x.reshape(1, K).repeat(3, 1)
    Y = torch.empty((3, N), device="cuda")
    gemm_q_npu(comb, X, Y, B=3, N=N, K=K)
    after = ctx.info()
    assert after["handles"] == before["handles"] and after["allocs"] == before["allocs"]
    assert torch.equal(y1, y2) and torch.equal(Y[1], y1)
    comb.add_(0)   # an in-place torch change bumps the version: repacked again
    gemv_q_npu(comb, x, y2, N=N, K=K)
    assert ctx.info()["handles"] == after["handles"] + 1
    ops.clear_weight_cache()
