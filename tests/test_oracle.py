"""The CPU oracle pinned against fixtures produced by the reference's own code
(tests/golden/make_golden.py).  CPU only."""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import q4


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_bf16_bit_restatement_matches_ml_dtypes():
    rng = np.random.default_rng(3)
    a = np.concatenate([
        rng.normal(0, 1, 200000).astype(np.float32),
        rng.normal(0, 1e-38, 1000).astype(np.float32),      # subnormals
        np.array([0.0, -0.0, np.inf, -np.inf, 3.4e38, 1 + 2**-8, 1 + 3 * 2**-8], np.float32),
    ])
    np.testing.assert_array_equal(q4.bf16_round_f32(a).view(np.uint32),
                                  q4.to_bf16(a).view(np.uint32))


def test_quantizer_and_packer_match_reference(golden_dir):
    g = _load(golden_dir, "quant_64x256.npz")
    comb = q4.quantize_combined(g["W"])
    np.testing.assert_array_equal(comb, g["combined"])
    deq = q4.dequantize_combined(g["combined"])
    np.testing.assert_array_equal(deq.view(np.uint32) >> 16, g["deq_bits"].astype(np.uint32))
    # zero block -> scale 1.0 (gemv_q_convert.py:27-28)
    q, sb = q4.unpack_combined(comb)
    assert sb[3, 0] == 0x3F80 and np.all(q[3, :32] == 0)


def test_dequant_random_bytes_match_reference(golden_dir):
    g = _load(golden_dir, "randbytes_48x256.npz")
    deq = q4.dequantize_combined(g["combined"])
    np.testing.assert_array_equal(deq.view(np.uint32) >> 16, g["deq_bits"].astype(np.uint32))
    q, _ = q4.unpack_combined(g["combined"])
    assert q.min() == -8 and q.max() == 7
    y = q4.gemv_q(g["combined"], g["x"])
    np.testing.assert_allclose(y, g["y32"], rtol=1e-5, atol=1e-5)


def test_reference_unit_test_case(golden_dir):
    """tests/test_gemv_q.py:76-94 of the reference (256x256, uniform, seed 42)."""
    g = _load(golden_dir, "ref_test_tiny_256.npz")
    np.testing.assert_array_equal(q4.quantize_combined(g["W"]), g["combined"])
    xb = q4.to_bf16(g["x"])
    y = q4.gemv_q(g["combined"], xb)
    np.testing.assert_allclose(y, g["y32"], rtol=1e-5, atol=1e-4)
    # the reference's bf16 output: equal except at float-order rounding ties
    yb = q4.bf16_bits(y)
    assert np.mean(yb == g["y_bf16_bits"]) > 0.97


@pytest.mark.parametrize("act", ["gelu", "silu"])
def test_ffn_matches_reference_expressions(golden_dir, act):
    g = _load(golden_dir, "ffn_256x512.npz")
    y, a, gate, up = q4.ffn(g["gate_c"], g["up_c"], g["down_c"], g["x"], act)
    np.testing.assert_array_equal(q4.bf16_bits(gate), g["gate_bits"])
    np.testing.assert_array_equal(q4.bf16_bits(up), g["up_bits"])
    np.testing.assert_array_equal(q4.bf16_bits(a), g[f"act_{act}_bits"])
    np.testing.assert_allclose(y, g[f"y_{act}32"], rtol=1e-5, atol=1e-4)


def test_gemm_matches_reference(golden_dir):
    g = _load(golden_dir, "gemm_5x96x256.npz")
    X = q4.bits_to_f32(g["X_bits"])
    Y = q4.gemm_q(g["combined"], X)
    np.testing.assert_allclose(Y, g["Y32"], rtol=1e-5, atol=1e-4)


def test_config1_full_size_hashes(golden_dir):
    """BASELINE config 1 (6912x1152, seed 0): the quantized bytes are
    bit-identical to the reference's and the bf16 output hash matches."""
    h = json.loads(open(os.path.join(golden_dir, "hashes.json")).read())
    rng = np.random.default_rng(0)
    W = rng.normal(0, 0.02, (6912, 1152)).astype(np.float32)
    x = rng.normal(0, 1, 1152).astype(np.float32)
    comb = q4.quantize_combined(W)
    assert hashlib.sha256(comb.tobytes()).hexdigest() == h["config1_combined"]
    y = q4.gemv_q(comb, x)
    assert abs(float(np.sum(y.astype(np.float64))) - h["config1_y32_sum"]) < 1e-3
