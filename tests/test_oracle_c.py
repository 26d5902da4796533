"""The C restatement of the oracle (oracle/q4_cpu.c) agrees with the numpy
oracle and with the reference goldens.  CPU only."""
import os

import numpy as np
import pytest

from oracle import cpu, q4


def normwise(y, ref):
    return float(np.max(np.abs(np.float64(y) - ref)) / max(np.max(np.abs(ref)), 1e-30))


def test_c_gemv_matches_reference_golden(golden_dir):
    g = np.load(os.path.join(golden_dir, "randbytes_48x256.npz"))
    assert normwise(cpu.gemv(g["combined"], g["x"]), g["y32"]) < 1e-5


def test_c_gemv_config1_matches_numpy_oracle():
    rng = np.random.default_rng(0)
    comb = q4.quantize_combined(rng.normal(0, 0.02, (6912, 1152)).astype(np.float32))
    x = rng.normal(0, 1, 1152).astype(np.float32)
    assert normwise(cpu.gemv(comb, x), q4.gemv_q(comb, x)) < 1e-5


@pytest.mark.parametrize("act", ["gelu", "silu"])
def test_c_ffn_matches_reference_golden(golden_dir, act):
    g = np.load(os.path.join(golden_dir, "ffn_256x512.npz"))
    y, a = cpu.ffn(g["gate_c"], g["up_c"], g["down_c"], g["x"], act)
    ref_act = q4.bits_to_f32(g[f"act_{act}_bits"])
    assert np.mean(a == ref_act) > 0.99   # act is bf16: equal except at rounding ties
    assert normwise(y, g[f"y_{act}32"]) < 1e-3


def test_c_ffn_block_matches_numpy_oracle():
    rng = np.random.default_rng(4)
    H, I = 256, 768
    cg = q4.quantize_combined(rng.normal(0, 0.02, (I, H)).astype(np.float32))
    cu = q4.quantize_combined(rng.normal(0, 0.02, (I, H)).astype(np.float32))
    cd = q4.quantize_combined(rng.normal(0, 0.02, (H, I)).astype(np.float32))
    x = q4.to_bf16(rng.normal(0, 1, H).astype(np.float32))
    ref = q4.ffn_block_gemma4(x, cg, cu, cd)
    got = cpu.ffn_block(cg, cu, cd, x)
    assert normwise(got, ref) < 1e-2 and np.mean(got == ref) > 0.95


def test_c_multithreaded_equals_single_thread():
    rng = np.random.default_rng(5)
    comb = q4.quantize_combined(rng.normal(0, 0.02, (512, 1024)).astype(np.float32))
    x = rng.normal(0, 1, 1024).astype(np.float32)
    np.testing.assert_array_equal(cpu.gemv(comb, x, 1), cpu.gemv(comb, x, 4))
