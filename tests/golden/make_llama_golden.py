"""Golden greedy tokens of BASELINE config 3, produced by the REFERENCE's own
Llama CPU path.

    ALVEARE_REFERENCE=/path/to/alveare python tests/golden/make_llama_golden.py [--steps 256]

Builds the random-init Q4 Llama-3.2-1B-shaped model of BASELINE config 3
(``oracle.llama.synthetic_weights``, seed 0, quantized with the reference's
own ``quantize_to_q4_0`` + ``pack_to_combined``), loads it into the
reference's ``LlamaNPUModel`` (runtime/py/model.py) -- the object is filled
in directly, since its constructor loads from disk and sets up the NPU --
and runs the reference's greedy loop (tests/test_generation.py:72-99: the
prompt token by token with ``forward(..., use_npu=False)``, then argmax).
The NPU toolchain (``aie``) and the NPU kernel modules are absent here;
stand-in modules satisfy model.py's imports and are never called on the
``use_npu=False`` path.

The same run is repeated with the numpy restatement ``oracle.llama`` and the
two must agree bit for bit (tokens and every step's logits).  Writes
``tests/golden/llama_config3.json``: the prompt, the greedy tokens, each
step's top-two logits and logits hash, and sha256 digests of the packed
weights, so a GPU test can rebuild the same model and check it.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import os
import sys
import time
import types
from pathlib import Path

import numpy as np
from ml_dtypes import bfloat16

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import llama  # noqa: E402

OUT = Path(__file__).resolve().parent / "llama_config3.json"


def _reference_root() -> Path:
    root = os.environ.get("ALVEARE_REFERENCE")
    if not root:
        raise SystemExit("set ALVEARE_REFERENCE to the root of a checkout of the reference project")
    return Path(root)


class _Absent:
    """Stand-in for the NPU toolchain's objects: any attribute or call gives
    another stand-in; used as a decorator it returns the function."""

    def __init__(self, *a, **k):
        pass

    def __call__(self, *a, **k):
        if len(a) == 1 and callable(a[0]) and not k:
            return a[0]
        return _Absent()

    def __getattr__(self, name):
        return _Absent()


def _absent_module(name: str):
    m = types.ModuleType(name)
    m.__getattr__ = lambda n: _Absent()  # PEP 562
    sys.modules[name] = m
    return m


def load_reference_model_class(ref: Path):
    for name in ("aie", "aie.iron", "aie.utils", "aie.utils.compile", "aie.utils.compile.jit",
                 "aie.utils.compile.jit.compilabledesign", "kernels", "kernels.gemv_q", "kernels.gemv_q.gemv_q",
                 "kernels.gemm_q", "kernels.gemm_q.gemm_q", "kernels.rmsnorm", "kernels.rmsnorm.rmsnorm",
                 "kernels.rope", "kernels.rope.rope", "kernels.ffn_fused", "kernels.ffn_fused.ffn_fused"):
        _absent_module(name)
    sys.path.insert(0, str(ref))
    spec = importlib.util.spec_from_file_location("alveare_reference_model", ref / "runtime" / "py" / "model.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.LlamaNPUModel


def reference_quantizer(ref: Path):
    sys.path.insert(0, str(ref))
    from tools.convert.gemv_q_convert import pack_to_combined, quantize_to_q4_0

    def quantize(W):
        return pack_to_combined(*quantize_to_q4_0(W))
    return quantize


def build_reference_model(cls, cfg: llama.Config, w: dict, ref: Path):
    from tools.ref.gemv_q import dequantize_combined
    m = cls.__new__(cls)
    m.model_type = "llama"
    m.max_seq_len = cfg.max_seq
    m.hidden_size, m.intermediate_size = cfg.hidden, cfg.intermediate
    m.num_attention_heads, m.num_key_value_heads = cfg.heads, cfg.kv_heads
    m.head_dim, m.num_hidden_layers, m.vocab_size = cfg.head_dim, cfg.layers, cfg.vocab
    m.config = {}
    m.token_embd = w["token_embd"]
    m.output_norm = w["output_norm.weight"]
    m.layer_attn_norms = [w[f"blk.{l}.attn_norm.weight"] for l in range(cfg.layers)]
    m.layer_ffn_norms = [w[f"blk.{l}.ffn_norm.weight"] for l in range(cfg.layers)]
    # model.py:135-145
    m.layer_weights_dequant = [{p: dequantize_combined(w[f"blk.{l}.{p}.weight_packed"]).astype(bfloat16)
                                for p in llama.PROJ} for l in range(cfg.layers)]
    m.lm_head_dequant = dequantize_combined(w["lm_head_packed"]).astype(bfloat16)
    m.cos_sin_table = m.precompute_cos_sin_table()
    m.k_caches = [np.zeros((cfg.kv_heads, cfg.max_seq, cfg.head_dim), dtype=bfloat16) for _ in range(cfg.layers)]
    m.v_caches = [np.zeros((cfg.kv_heads, cfg.max_seq, cfg.head_dim), dtype=bfloat16) for _ in range(cfg.layers)]
    return m


def reference_generate(m, prompt, steps):
    """tests/test_generation.py:72-99 with the CPU path and no EOS stop."""
    m.reset_caches()
    for pos in range(len(prompt) - 1):
        m.forward(int(prompt[pos]), pos, return_logits=False, use_npu=False)
    tok, pos = int(prompt[-1]), len(prompt) - 1
    toks, logits = [], []
    for _ in range(steps):
        lg = m.forward(tok, pos, use_npu=False)
        tok = int(np.argmax(lg))
        toks.append(tok)
        logits.append(lg)
        pos += 1
    return toks, logits


def weights_digest(w: dict, cfg: llama.Config) -> dict:
    out = {"lm_head_packed": hashlib.sha256(w["lm_head_packed"].tobytes()).hexdigest(),
           "token_embd": hashlib.sha256(w["token_embd"].tobytes()).hexdigest()}
    h = hashlib.sha256()
    for l in range(cfg.layers):
        for p in llama.PROJ:
            h.update(w[f"blk.{l}.{p}.weight_packed"].tobytes())
    out["layers_packed"] = h.hexdigest()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    ref = _reference_root()
    cfg = llama.Config(max_seq=512)
    t0 = time.time()
    w, prompt = llama.synthetic_weights(cfg, args.seed, quantize=reference_quantizer(ref))
    print(f"weights {time.time() - t0:.0f} s", flush=True)
    cls = load_reference_model_class(ref)
    m = build_reference_model(cls, cfg, w, ref)
    t0 = time.time()
    toks, logits = reference_generate(m, prompt, args.steps)
    print(f"reference run {time.time() - t0:.0f} s", flush=True)
    del m
    orc = llama.LlamaOracle(cfg, w)
    t0 = time.time()
    o_toks, o_logits = orc.generate(prompt, args.steps, keep_logits=True)
    print(f"oracle run {time.time() - t0:.0f} s", flush=True)
    agree_tokens = o_toks == toks
    agree_logits = all(np.array_equal(a, b) for a, b in zip(o_logits, logits))
    steps = []
    for lg in logits:
        i, mx, second = llama.top2_gap(lg)
        steps.append({"token": i, "max": mx, "second": second,
                      "logits_sha256": hashlib.sha256(lg.astype(bfloat16).tobytes()).hexdigest()})
    doc = {
        "what": "BASELINE config 3: greedy decode of a random-init Q4 Llama-3.2-1B-shaped model, produced by "
                "the reference's LlamaNPUModel.forward(use_npu=False) (runtime/py/model.py:821-934) and its "
                "greedy loop (tests/test_generation.py:72-99)",
        "seed": args.seed, "config": vars(cfg), "prompt": [int(t) for t in prompt], "tokens": toks,
        "steps": steps, "weights_sha256": weights_digest(w, cfg),
        "oracle_restatement_agrees": {"tokens": bool(agree_tokens), "logits_bitwise": bool(agree_logits)},
        "kv_cache_dtype": "bf16 (the reference's cache, runtime/py/model.py:173-174)",
    }
    OUT.write_text(json.dumps(doc, indent=1) + "\n")
    print(f"wrote {OUT}; oracle agrees: tokens {agree_tokens}, logits {agree_logits}")


if __name__ == "__main__":
    main()
