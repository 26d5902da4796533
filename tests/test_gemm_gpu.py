"""Batched prefill gemm_q on the tcgen05 tensor cores (alv_gemm) against the
oracle (kernels/gemm_q/gemm_q.py:185-188: X_f32 @ dequantize_combined(W).T)
and against an fp32 matmul of the GPU's own dequantized weights.  Tolerance
(north star): max|y - y_ref| / max|y_ref| <= 1e-3 on fp32 outputs."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from alveare_b200 import Q4Weight, gemm_q_npu, q4_quantize  # noqa: E402
from alveare_b200 import _lib  # noqa: E402
from oracle import q4  # noqa: E402

TOL = 1e-3


def normwise(y, ref):
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(y - ref)) / max(np.max(np.abs(ref)), 1e-30))


def run_gemm(w, x_bf16: torch.Tensor, y_dtype=torch.float32):
    B = x_bf16.shape[0]
    y = torch.empty((B, w.N), dtype=y_dtype, device="cuda")
    ctx = w.ctx
    ctx.check(ctx.lib.alv_gemm(ctx.ptr, w.handle, B, x_bf16.data_ptr(), y.data_ptr(),
                               _lib.F32 if y_dtype == torch.float32 else _lib.BF16,
                               torch.cuda.current_stream().cuda_stream), "alv_gemm")
    ctx.sync_status()
    return y


def dequantized(w):
    """The GPU's bf16 dequantization of w (bit-exact with the reference)."""
    out = torch.empty((w.N, w.K), dtype=torch.bfloat16, device="cuda")
    ctx = w.ctx
    ctx.check(ctx.lib.alv_weight_dequantize(ctx.ptr, w.handle, 0, out.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream), "dequantize")
    ctx.sync_status()
    return out.float()


def test_gemm_reference_golden(golden_dir):
    """B=5, N=96, K=256 fixture evaluated with the reference's dequantize_combined."""
    d = np.load(os.path.join(golden_dir, "gemm_5x96x256.npz"))
    w = Q4Weight(d["combined"])
    x = torch.from_numpy(d["X_bits"].view(np.int16)).cuda().view(torch.bfloat16)
    y = run_gemm(w, x).cpu().numpy()
    assert normwise(y, d["Y32"]) <= TOL
    w.free()


@pytest.mark.parametrize("N,K,B", [(256, 256, 17), (1000, 512, 300), (4096, 2048, 257), (192, 3840, 64)])
def test_gemm_shapes_against_fp32_matmul(N, K, B):
    g = torch.Generator(device="cuda").manual_seed(N + K + B)
    w = Q4Weight(q4_quantize(torch.randn((N, K), generator=g, device="cuda") * 0.02))
    x = torch.randn((B, K), generator=g, device="cuda").to(torch.bfloat16)
    y = run_gemm(w, x)
    ref = x.float() @ dequantized(w).T
    assert normwise(y.cpu().numpy(), ref.cpu().numpy()) <= 1e-4
    yb = run_gemm(w, x, torch.bfloat16)
    assert torch.equal(yb, y.to(torch.bfloat16))
    w.free()


def test_gemm_config5_prefill_against_oracle():
    """X (512 x 3840) bf16, W (15360 x 3840) Q4, checked
    against the oracle on 1024 of the 15360 output rows: three whole 128-row
    tensor-core tiles (first, middle, last) and 640 rows drawn at random."""
    rng = np.random.default_rng(0)
    N, K, B = 15360, 3840, 512
    Wf = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    comb = q4.quantize_combined(Wf)
    X = q4.to_bf16(rng.normal(0, 1, (B, K)).astype(np.float32))
    w = Q4Weight(comb)
    x = torch.from_numpy(q4.bf16_bits(X).view(np.int16)).cuda().view(torch.bfloat16)
    y = run_gemm(w, x).cpu().numpy()
    tiles = np.concatenate([np.arange(0, 128), np.arange(7680, 7808), np.arange(N - 128, N)])
    rest = np.setdiff1d(np.arange(N), tiles)
    rows = np.sort(np.concatenate([tiles, rng.choice(rest, 640, replace=False)]))
    assert len(rows) == 1024
    ref = q4.gemm_q(comb[rows], X)
    assert normwise(y[:, rows], ref) <= TOL
    full = (x.float() @ dequantized(w).T).cpu().numpy()
    assert normwise(y, full) <= 1e-4
    w.free()


def test_gemm_generic_dequant_path():
    """Scales spanning more than the fast window select the generic dequant."""
    rng = np.random.default_rng(5)
    N, K, B = 128, 512, 40
    comb = q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    v = comb.reshape(N, K // 32, 20)
    v[0, 0, 16:18] = [0x00, 0x01]   # 2^-125
    v[1, 0, 16:18] = [0x80, 0x40]   # 4.0
    w = Q4Weight(comb)
    assert w.info()[3] == 0
    X = q4.to_bf16(rng.normal(0, 1, (B, K)).astype(np.float32))
    x = torch.from_numpy(q4.bf16_bits(X).view(np.int16)).cuda().view(torch.bfloat16)
    y = run_gemm(w, x).cpu().numpy()
    assert normwise(y, q4.gemm_q(comb, X)) <= TOL
    w.free()


def test_gemm_q_npu_routes_large_bf16_batches_to_the_tensor_cores():
    """gemm_q_npu: 48 bf16 tokens (tensor cores) give the same result as the
    same tokens pushed through the streaming gemv 16 at a time."""
    g = torch.Generator(device="cuda").manual_seed(9)
    N, K, B = 512, 1024, 48
    comb = q4_quantize(torch.randn((N, K), generator=g, device="cuda") * 0.02)
    w = Q4Weight(comb)
    x = torch.randn((B, K), generator=g, device="cuda").to(torch.bfloat16)
    y_tc = torch.empty((B, N), dtype=torch.float32, device="cuda")
    gemm_q_npu(w, x, y_tc, B=B, N=N, K=K)
    y_gemv = torch.empty((B, N), dtype=torch.float32, device="cuda")
    for b0 in range(0, B, 16):
        gemm_q_npu(w, x[b0:b0 + 16], y_gemv[b0:b0 + 16], B=16, N=N, K=K)
    torch.cuda.synchronize()
    assert normwise(y_tc.cpu().numpy(), y_gemv.cpu().numpy()) <= 1e-4
    w.free()
