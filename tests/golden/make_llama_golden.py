"""Golden greedy tokens of BASELINE config 3, produced by the REFERENCE's own
Llama CPU path.

    ALVEARE_REFERENCE=/path/to/alveare python tests/golden/make_llama_golden.py [--steps 256]
    ALVEARE_REFERENCE=/path/to/alveare python tests/golden/make_llama_golden.py --small

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

``--small`` runs the reference's greedy loop on small models of the same
family (SMALL_CASES: other FFN widths, vocabularies and prompts) and
writes ``tests/golden/llama_small.npz`` with every step's full bf16 logits,
so the CPU test suite checks the numpy restatement against the reference
itself in seconds.
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
OUT_SMALL = Path(__file__).resolve().parent / "llama_small.npz"

# Small models for the CPU-side pin of oracle/llama.py: (name, Config
# arguments, weight seed, prompt length, greedy steps).  The reference's CPU
# path fixes the Llama-3.2-1B attention shapes and depth (runtime/py/
# model.py:821-837, 921: 16 layers, 32 query heads and 8 KV heads of 64,
# hidden 2048), so the cases vary the FFN width, the vocabulary and the
# prompt length around them.
SMALL_CASES = (
    ("i512_v1024", dict(intermediate=512, vocab=1024, vocab_padded=1024, max_seq=64), 11, 24, 16),
    ("i1536_v2048", dict(intermediate=1536, vocab=2048, vocab_padded=2048, max_seq=64), 5, 40, 12),
)


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


def bf16_bits(a) -> np.ndarray:
    return np.asarray(a, np.float32).astype(bfloat16).view(np.uint16)


def make_small(ref: Path):
    """The reference's greedy loop on each of SMALL_CASES; every step's full
    logits (bf16 bits) into llama_small.npz, after checking that the numpy
    restatement gives the same bits."""
    cls = load_reference_model_class(ref)
    quantize = reference_quantizer(ref)
    out = {}
    for name, kw, seed, n_prompt, steps in SMALL_CASES:
        cfg = llama.Config(**kw)
        w, prompt = llama.synthetic_weights(cfg, seed, quantize=quantize)
        prompt = prompt[:n_prompt]
        m = build_reference_model(cls, cfg, w, ref)
        toks, logits = reference_generate(m, prompt, steps)
        o_toks, o_logits = llama.LlamaOracle(cfg, w).generate(prompt, steps, keep_logits=True)
        agree = o_toks == toks and all(np.array_equal(bf16_bits(a), bf16_bits(b)) for a, b in zip(o_logits, logits))
        print(f"{name}: tokens {toks}; oracle agrees: {agree}")
        if not agree:
            raise SystemExit(f"{name}: the restatement differs from the reference")
        out[f"{name}.config"] = np.array(json.dumps(kw))
        out[f"{name}.seed"] = np.array(seed)
        out[f"{name}.prompt"] = np.asarray(prompt, np.int64)
        out[f"{name}.tokens"] = np.asarray(toks, np.int64)
        out[f"{name}.logits_bf16"] = np.stack([bf16_bits(lg) for lg in logits])
        out[f"{name}.weights_sha256"] = np.array(json.dumps(weights_digest(w, cfg)))
    np.savez_compressed(OUT_SMALL, **out)
    print(f"wrote {OUT_SMALL}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--small", action="store_true", help="write llama_small.npz (SMALL_CASES) instead")
    args = ap.parse_args()
    ref = _reference_root()
    if args.small:
        make_small(ref)
        return
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
