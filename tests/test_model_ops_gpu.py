"""Model-level wrappers (alveare_b200.model_ops.GpuModelOps) against the
reference's LlamaNPUModel contract (runtime/py/model.py:283-485): same
arguments (packed weights, bf16 host x, zero-padded to K), bf16 host results,
and values equal to the oracle's fp32 result rounded to bf16 up to one bf16
rounding step (1e-3 normwise in fp32, the north star's tolerance)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from alveare_b200.model_ops import GpuModelOps  # noqa: E402
from oracle import q4  # noqa: E402


def normwise(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    return float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))


def test_run_gemv_npu_pads_x_and_keeps_weights_resident():
    rng = np.random.default_rng(11)
    N, K = 300, 512
    comb = q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    x = q4.to_bf16(rng.normal(0, 1, K - 64).astype(np.float32))   # shorter than K: zero-padded
    ops = GpuModelOps()
    y = ops.run_gemv_npu(comb, x.astype(q4.bfloat16))
    assert y.dtype.name == "bfloat16" and y.shape == (N,)
    xp = np.zeros(K, np.float32)
    xp[:K - 64] = x
    ref = q4.gemv_q(comb, xp)
    assert normwise(y.astype(np.float32), ref) <= 4e-3   # one bf16 rounding of y
    assert np.array_equal(y.astype(np.float32), q4.to_bf16(y.astype(np.float32)))
    y2 = ops.run_gemv_npu(comb, x.astype(q4.bfloat16))
    assert len(ops._resident) == 1 and np.array_equal(y, y2)
    ops.free()


@pytest.mark.parametrize("act", ["gelu", "silu"])
def test_run_ffn_fused_npu_matches_oracle(act):
    rng = np.random.default_rng(12)
    H, I = 256, 1024
    cg, cu = (q4.quantize_combined(rng.normal(0, 0.02, (I, H)).astype(np.float32)) for _ in range(2))
    cd = q4.quantize_combined(rng.normal(0, 0.02, (H, I)).astype(np.float32))
    x = q4.to_bf16(rng.normal(0, 1, H).astype(np.float32))
    ops = GpuModelOps(activation=act)
    ops.register_ffn_layer(3, cg, cu, cd, H, I)
    y = ops.run_ffn_fused_npu(3, x.astype(q4.bfloat16))
    assert y.dtype.name == "bfloat16" and y.shape == (H,)
    ref, _, _, _ = q4.ffn(cg, cu, cd, x, act)
    assert normwise(y.astype(np.float32), ref) <= 4e-3
    with pytest.raises(KeyError):
        ops.run_ffn_fused_npu(4, x.astype(q4.bfloat16))
    ops.free()


@pytest.mark.parametrize("B", [5, 40])
def test_run_gemm_npu_matches_oracle(B):
    rng = np.random.default_rng(13 + B)
    N, K = 192, 512
    comb = q4.quantize_combined(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    X = q4.to_bf16(rng.normal(0, 1, (B, K)).astype(np.float32))
    ops = GpuModelOps()
    Y = ops.run_gemm_npu(comb, X.astype(q4.bfloat16))
    assert Y.dtype.name == "bfloat16" and Y.shape == (B, N)
    assert normwise(Y.astype(np.float32), q4.gemm_q(comb, X)) <= 4e-3
    ops.free()
