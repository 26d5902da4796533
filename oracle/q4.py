"""CPU oracle for the Q4 decode hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain numpy, the reference's CPU arithmetic for the
Q4 block format, the quantized GEMV, the fused FFN and the batched gemm.  It is
the checker the CUDA path is compared against.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it;
the product path (``alveare_b200``) never does.

Every function cites the reference file:line it restates (paths inside the
daino-selvatico/alveare project).  The restatement is pinned against the
reference itself by ``tests/golden/make_golden.py``, which imports the
reference's own ``tools/convert/gemv_q_convert.py`` and ``tools/ref/gemv_q.py``
to produce the committed fixtures that ``tests/test_oracle.py`` checks.

bf16 casts use ``ml_dtypes.bfloat16`` (the same library and therefore the same
rounding as the reference: float32 -> bf16 is round-to-nearest-even, and
float64 -> bf16 goes through float32 first).  ``bf16_round_f32`` is an
independent bit-level restatement of the C++ runtime's RNE conversion
(runtime/cpp/src/bf16.cpp:7-18) used to cross-check it.
"""
from __future__ import annotations

import numpy as np
from ml_dtypes import bfloat16

BLOCK = 32          # weights per Q4 block along K (gemv_q_convert.py:17-21)
BLOCK_BYTES = 20    # 16 B nibbles + 2 B bf16 scale + 2 B pad (gemv_q_convert.py:58-61)


# ----------------------------------------------------------------------------
# bf16 helpers
# ----------------------------------------------------------------------------
def to_bf16(a) -> np.ndarray:
    """Round to bf16 exactly as the reference's ``.astype(bfloat16)`` does and
    return the result widened back to float32."""
    return np.asarray(a).astype(bfloat16).astype(np.float32)


def bf16_round_f32(a: np.ndarray) -> np.ndarray:
    """Bit-level float32 -> bf16 round-to-nearest-even, widened back to float32.

    Restates runtime/cpp/src/bf16.cpp:7-18 (NaN -> quiet NaN 0x7FC0, else add
    0x7FFF + lsb and truncate)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(np.isnan(a), 0x7FC0, r).astype(np.uint32)
    return (r << 16).view(np.float32).reshape(a.shape)


def bf16_bits(a) -> np.ndarray:
    """bf16 bit patterns (uint16) of ``a`` rounded as the reference rounds."""
    return np.asarray(a).astype(bfloat16).view(np.uint16)


def bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen bf16 bit patterns (uint16) to float32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------
# Q4 format: quantize, pack, dequantize
# ----------------------------------------------------------------------------
def quantize_to_q4_0(W: np.ndarray):
    """Q4_0 quantizer.  Restates tools/convert/gemv_q_convert.py:5-51.

    Per row and per 32-block along K: ``scale = max|w| / 7`` in float32, zero
    scales replaced by 1.0 (:24-28); ``q = clip(rint(w / scale), -8, 7)`` with
    numpy's round-half-to-even on the float32 quotient (:34-37); nibble pack,
    even k in the low nibble, odd k in the high nibble (:45-48).

    Returns ``(w_q4 uint8 (N, K/2), scale_bits uint16 (N, K/32))`` -- the
    scale is returned as its bf16 bit pattern (the reference returns a bf16
    array, :51).
    """
    W = np.asarray(W)
    N, K = W.shape
    if K % BLOCK:
        raise ValueError(f"K must be a multiple of 32, got {K}")
    blocks = W.reshape(N, K // BLOCK, BLOCK)
    scales = np.max(np.abs(blocks), axis=2) / 7.0
    scales[scales == 0.0] = 1.0
    q = np.round(blocks / scales[:, :, None]).astype(np.int32)
    q = np.clip(q, -8, 7).reshape(N, K)
    w_q4 = ((q[:, 0::2] & 0x0F) | ((q[:, 1::2] & 0x0F) << 4)).astype(np.uint8)
    return w_q4, bf16_bits(scales)


def pack_to_combined(w_q4: np.ndarray, scale_bits: np.ndarray) -> np.ndarray:
    """20-byte block packer.  Restates tools/convert/gemv_q_convert.py:53-85:
    per block, bytes 0-15 = nibbles, bytes 16-17 = bf16 scale little-endian,
    bytes 18-19 = 0.  Output (N, K/32*20) uint8."""
    N, K_half = w_q4.shape
    kb = (K_half * 2) // BLOCK
    out = np.zeros((N, kb, BLOCK_BYTES), dtype=np.uint8)
    out[:, :, :16] = w_q4.reshape(N, kb, 16)
    sb = np.asarray(scale_bits, dtype=np.uint16).reshape(N, kb)
    out[:, :, 16] = (sb & 0xFF).astype(np.uint8)
    out[:, :, 17] = (sb >> 8).astype(np.uint8)
    return out.reshape(N, kb * BLOCK_BYTES)


def quantize_combined(W: np.ndarray) -> np.ndarray:
    """quantize_to_q4_0 followed by pack_to_combined (the producer path of
    tools/quantize_gemma4.py:177-189)."""
    return pack_to_combined(*quantize_to_q4_0(W))


def unpack_combined(combined: np.ndarray):
    """Split the (N, K/32*20) layout into signed int8 q (N, K) and the bf16
    scale bit patterns (N, K/32).  Restates tools/ref/gemv_q.py:39-62 and the
    nibble decode of :15-29."""
    combined = np.ascontiguousarray(combined, dtype=np.uint8)
    N, nb = combined.shape
    kb = nb // BLOCK_BYTES
    r = combined.reshape(N, kb, BLOCK_BYTES)
    nib = r[:, :, :16].reshape(N, kb * 16)
    scale_bits = r[:, :, 16].astype(np.uint16) | (r[:, :, 17].astype(np.uint16) << 8)
    q0 = (nib & 0x0F).astype(np.int8)
    q1 = ((nib >> 4) & 0x0F).astype(np.int8)
    q0[q0 >= 8] -= 16
    q1[q1 >= 8] -= 16
    q = np.empty((N, kb * BLOCK), dtype=np.int8)
    q[:, 0::2] = q0
    q[:, 1::2] = q1
    return q, scale_bits


def dequantize_combined(combined: np.ndarray) -> np.ndarray:
    """Dequantize to bf16-valued float32 (N, K).  Restates
    tools/ref/gemv_q.py:4-62: ``w = bf16(float32(q) * float32(scale))``."""
    q, scale_bits = unpack_combined(combined)
    s = np.repeat(bits_to_f32(scale_bits), BLOCK, axis=1)
    return to_bf16(q.astype(np.float32) * s)


# ----------------------------------------------------------------------------
# GEMV / GEMM
# ----------------------------------------------------------------------------
def gemv_q(combined: np.ndarray, x: np.ndarray, w_deq: np.ndarray | None = None) -> np.ndarray:
    """Quantized GEMV in float32 before the final bf16 cast.  Restates
    tools/ref/gemv_q.py:73-80 (``dequantize_combined(W).astype(f32) @
    x.astype(f32)``).  ``x`` may be (K,) or (B, K); returns (N,) or (B, N)."""
    W = dequantize_combined(combined) if w_deq is None else w_deq
    x = np.asarray(x, dtype=np.float32)
    if x.ndim == 1:
        return W @ x
    return x @ W.T


def gemm_q(combined: np.ndarray, X: np.ndarray, w_deq: np.ndarray | None = None) -> np.ndarray:
    """Batched prefill matmul ``Y[B,N] = X[B,K] @ W_deq^T`` in float32.
    Restates kernels/gemm_q/gemm_q.py:185-188 with the bf16 X widened to f32."""
    W = dequantize_combined(combined) if w_deq is None else w_deq
    return np.asarray(X, dtype=np.float32) @ W.T


# ----------------------------------------------------------------------------
# Fused FFN
# ----------------------------------------------------------------------------
def act_geglu(gate_bf: np.ndarray, up_bf: np.ndarray) -> np.ndarray:
    """GeGLU, bf16 result.  Restates runtime/py/model.py:690-693 (gemma3) and
    :798-801 (gemma4) with numpy's exact promotion: the inner cubic term is
    float32, the ``np.sqrt(2/pi)`` factor is a numpy float64 scalar so tanh and
    everything after it are float64, and the float64 -> bf16 cast goes through
    float32 (ml_dtypes)."""
    g = gate_bf.astype(np.float32)
    u = up_bf.astype(np.float32)
    gelu = 0.5 * g * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (g + 0.044715 * (g ** 3))))
    return to_bf16(gelu * u)


def act_swiglu(gate_bf: np.ndarray, up_bf: np.ndarray) -> np.ndarray:
    """SwiGLU, bf16 result.  Restates runtime/py/model.py:857-859 (all
    float32: ``g * (1 / (1 + exp(-g))) * u``)."""
    g = gate_bf.astype(np.float32)
    u = up_bf.astype(np.float32)
    return to_bf16((g * (1.0 / (1.0 + np.exp(-g)))) * u)


def ffn(gate_c, up_c, down_c, x, activation: str = "gelu", deq=None):
    """Fused FFN with the reference CPU path's bf16 rounding points.

    Restates runtime/py/model.py:687-698 (GeGLU) / :854-860 (SwiGLU):
    ``gate = bf16(Wg x)``, ``up = bf16(Wu x)``, ``act = bf16(act_fn(gate) *
    up)``, ``y = Wd act``.  Returns ``(y_f32, act, gate, up)`` where ``y_f32``
    is the float32 down projection before the reference's final bf16 cast.
    ``x`` may be (H,) or (B, H).  ``deq`` optionally supplies the three
    dequantized matrices to skip re-dequantizing.
    """
    if deq is None:
        deq = tuple(dequantize_combined(c) for c in (gate_c, up_c, down_c))
    Wg, Wu, Wd = deq
    x = np.asarray(x, dtype=np.float32)
    gate = to_bf16(gemv_q(None, x, Wg))
    up = to_bf16(gemv_q(None, x, Wu))
    if activation == "gelu":
        act = act_geglu(gate, up)
    elif activation == "silu":
        act = act_swiglu(gate, up)
    else:
        raise ValueError(f"unknown activation {activation!r}")
    y = gemv_q(None, act, Wd)
    return y, act, gate, up


# ----------------------------------------------------------------------------
# Layer glue around the FFN (used by the FFN-stack workload)
# ----------------------------------------------------------------------------
def rmsnorm_gemma(x_bf: np.ndarray, w: np.ndarray | None = None, eps: float = 1e-6) -> np.ndarray:
    """Gemma RMSNorm, bf16 result.  Restates runtime/py/model.py:522-529:
    float32 mean of squares, ``x * (1 / sqrt(var + eps))`` (times ``w`` when
    given), cast to bf16."""
    xf = np.asarray(x_bf, dtype=np.float32)
    var = np.mean(xf ** 2)
    normed = xf * (1.0 / np.sqrt(var + eps))
    if w is not None:
        normed = normed * w
    return to_bf16(normed)


def ffn_block_gemma4(x_bf: np.ndarray, gate_c, up_c, down_c, deq=None, activation: str = "gelu") -> np.ndarray:
    """One FFN half-block of a Gemma-4 decode layer with unit norm weights.
    Restates runtime/py/model.py:782-810 minus the layer output scale:
    ``x2 = rmsnorm(x)``; ``down = bf16(FFN_geglu(x2))``; ``x + bf16(rmsnorm(down))``
    with a bf16 residual add.  ``activation="silu"`` swaps in the SwiGLU FFN
    (model.py:854-860) inside the same block, for kernel checks."""
    x2 = rmsnorm_gemma(x_bf)
    y, _, _, _ = ffn(gate_c, up_c, down_c, x2, activation, deq=deq)
    down = to_bf16(y)
    down_normed = rmsnorm_gemma(down)
    return to_bf16(np.asarray(x_bf, dtype=np.float32) + down_normed)
