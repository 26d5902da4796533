"""Generate the committed golden fixtures by running the REFERENCE's own code.

Run where a checkout of the reference project is available (read-only) and
name its root in ``ALVEARE_REFERENCE``:

    ALVEARE_REFERENCE=/path/to/alveare python tests/golden/make_golden.py

It imports the reference's ``tools/convert/gemv_q_convert.py``
(``quantize_to_q4_0``, ``pack_to_combined``) and ``tools/ref/gemv_q.py``
(``dequantize_combined``, ``gemv_q_combined``) and writes small ``.npz``
fixtures plus ``hashes.json`` (sha256 of full-size outputs at the BASELINE
configs, so the big cases are pinned without committing megabytes).

The reference has no standalone FFN or gemm CPU function (the FFN math lives
inline in ``runtime/py/model.py:687-698, 854-860`` and the gemm check inline in
``kernels/gemm_q/gemm_q.py:185-188``); for those, this script evaluates the
same expressions on top of the reference's own ``dequantize_combined``.

Nothing at test time reads the reference: tests only read the files written
here.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
from ml_dtypes import bfloat16

OUT = Path(__file__).resolve().parent


def _reference_root() -> Path:
    root = os.environ.get("ALVEARE_REFERENCE")
    if not root:
        raise SystemExit("set ALVEARE_REFERENCE to the root of a checkout of the reference project")
    return Path(root)


def _ref():
    sys.path.insert(0, str(_reference_root()))
    from tools.convert.gemv_q_convert import pack_to_combined, quantize_to_q4_0
    from tools.ref.gemv_q import dequantize_combined, gemv_q_combined
    return quantize_to_q4_0, pack_to_combined, dequantize_combined, gemv_q_combined


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    quantize_to_q4_0, pack_to_combined, dequantize_combined, gemv_q_combined = _ref()

    def qc(W):
        q, s = quantize_to_q4_0(W)
        return pack_to_combined(q, s)

    # -- 1. quantizer + packer edge cases (zero block, exact .5 ties, negatives)
    rng = np.random.default_rng(0)
    W = rng.normal(0, 0.02, (64, 256)).astype(np.float32)
    W[3, 0:32] = 0.0                                  # zero block -> scale 1.0
    W[5, 32:64] = np.linspace(-7, 7, 32) / 7.0         # ties at k.5 after /scale
    W[7, 64:96] = np.arange(32, dtype=np.float32) - 16.0
    W[9, 96:128] = -1e-3                               # constant negative block
    comb = qc(W)
    deq = dequantize_combined(comb)
    np.savez_compressed(OUT / "quant_64x256.npz", W=W, combined=comb,
                        deq_bits=deq.view(np.uint16))

    # -- 2. random bytes (every nibble incl. -8), finite positive/negative scales
    rb = rng.integers(0, 256, (48, 8 * 20), dtype=np.uint8)
    sc = rng.normal(0, 0.05, (48, 8)).astype(np.float32).astype(bfloat16).view(np.uint16)
    rbv = rb.reshape(48, 8, 20)
    rbv[:, :, 16] = (sc & 0xFF).astype(np.uint8)
    rbv[:, :, 17] = (sc >> 8).astype(np.uint8)
    rbv[:, :, 18:] = 0
    rb = rbv.reshape(48, 160)
    x = rng.normal(0, 1, 256).astype(np.float32)
    y32 = dequantize_combined(rb).astype(np.float32) @ x
    np.savez_compressed(OUT / "randbytes_48x256.npz", combined=rb, x=x, y32=y32,
                        deq_bits=dequantize_combined(rb).view(np.uint16))

    # -- 3. the reference's own unit-test case: tests/test_gemv_q.py:76-94
    rng42 = np.random.default_rng(42)
    Wt = rng42.uniform(-1.0, 1.0, size=(256, 256)).astype(np.float32)
    xt = rng42.uniform(-1.0, 1.0, size=(256,)).astype(np.float32)
    ct = qc(Wt)
    yt = gemv_q_combined(ct, xt.astype(bfloat16))
    yt32 = dequantize_combined(ct).astype(np.float32) @ xt.astype(bfloat16).astype(np.float32)
    np.savez_compressed(OUT / "ref_test_tiny_256.npz", W=Wt, x=xt, combined=ct,
                        y_bf16_bits=yt.view(np.uint16), y32=yt32)

    # -- 4. FFN (GeGLU + SwiGLU) small case on the reference dequantizer
    H, I = 256, 512
    Wg = rng.normal(0, 0.02, (I, H)).astype(np.float32)
    Wu = rng.normal(0, 0.02, (I, H)).astype(np.float32)
    Wd = rng.normal(0, 0.02, (H, I)).astype(np.float32)
    xf = rng.normal(0, 1, H).astype(np.float32)
    cg, cu, cd = qc(Wg), qc(Wu), qc(Wd)
    dg, du, dd = (dequantize_combined(c) for c in (cg, cu, cd))
    # model.py:687-698 (GeGLU) and :854-860 (SwiGLU), evaluated verbatim in form
    gate = (dg.astype(np.float32) @ xf).astype(bfloat16)
    up = (du.astype(np.float32) @ xf).astype(bfloat16)
    gate_fp32 = gate.astype(np.float32)
    up_fp32 = up.astype(np.float32)
    gelu_out = 0.5 * gate_fp32 * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (gate_fp32 + 0.044715 * (gate_fp32 ** 3))))
    act_g = (gelu_out * up_fp32).astype(bfloat16)
    y_g = dd.astype(np.float32) @ act_g.astype(np.float32)
    silu_out = (gate_fp32 * (1.0 / (1.0 + np.exp(-gate_fp32)))) * up_fp32
    act_s = silu_out.astype(bfloat16)
    y_s = dd.astype(np.float32) @ act_s.astype(np.float32)
    np.savez_compressed(OUT / "ffn_256x512.npz", gate_c=cg, up_c=cu, down_c=cd, x=xf,
                        gate_bits=gate.view(np.uint16), up_bits=up.view(np.uint16),
                        act_gelu_bits=act_g.view(np.uint16), y_gelu32=y_g,
                        act_silu_bits=act_s.view(np.uint16), y_silu32=y_s)

    # -- 5. gemm (kernels/gemm_q/gemm_q.py:185-188) small case, bf16 X
    Wm = rng.normal(0, 0.02, (96, 256)).astype(np.float32)
    Xm = rng.normal(0, 1, (5, 256)).astype(np.float32).astype(bfloat16)
    cm = qc(Wm)
    Ym = Xm.astype(np.float32) @ dequantize_combined(cm).astype(np.float32).T
    np.savez_compressed(OUT / "gemm_5x96x256.npz", combined=cm, X_bits=Xm.view(np.uint16), Y32=Ym)

    # -- 6. full-size BASELINE configs, pinned by hash only
    hashes = {}
    rng0 = np.random.default_rng(0)
    W1 = rng0.normal(0, 0.02, (6912, 1152)).astype(np.float32)
    x1 = rng0.normal(0, 1, 1152).astype(np.float32)
    c1 = qc(W1)
    y1 = dequantize_combined(c1).astype(np.float32) @ x1
    hashes["config1_combined"] = sha(c1)
    hashes["config1_y_bf16"] = sha(gemv_q_combined(c1, x1).view(np.uint16))
    hashes["config1_y32_sum"] = float(np.sum(y1.astype(np.float64)))
    (OUT / "hashes.json").write_text(json.dumps(hashes, indent=1) + "\n")
    print("wrote goldens to", OUT)


if __name__ == "__main__":
    main()
