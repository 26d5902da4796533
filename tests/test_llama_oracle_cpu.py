"""The numpy restatement of the reference's Llama CPU decode path
(oracle/llama.py) against the reference itself: tests/golden/llama_small.npz
holds every greedy step's full bf16 logits from the reference's
LlamaNPUModel.forward(use_npu=False) (runtime/py/model.py:821-934) and its
greedy loop (tests/test_generation.py:72-99) on Llama-3.2-1B-shaped models
with a narrower FFN and a small vocabulary (made by
tests/golden/make_llama_golden.py --small).  The restatement must give the
same packed weights, the same tokens and the same logits bit for bit."""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import llama

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "llama_small.npz")


def _cases():
    with np.load(GOLDEN) as z:
        names = sorted({k.split(".")[0] for k in z.files})
        return [(n, {k.split(".", 1)[1]: z[k] for k in z.files if k.split(".")[0] == n}) for n in names]


def _digest(w: dict, cfg: llama.Config) -> dict:
    out = {"lm_head_packed": hashlib.sha256(w["lm_head_packed"].tobytes()).hexdigest(),
           "token_embd": hashlib.sha256(w["token_embd"].tobytes()).hexdigest()}
    h = hashlib.sha256()
    for l in range(cfg.layers):
        for p in llama.PROJ:
            h.update(w[f"blk.{l}.{p}.weight_packed"].tobytes())
    out["layers_packed"] = h.hexdigest()
    return out


@pytest.mark.parametrize("name,case", _cases(), ids=lambda v: v if isinstance(v, str) else "")
def test_restatement_matches_reference_logits(name, case):
    cfg = llama.Config(**json.loads(str(case["config"])))
    w, prompt = llama.synthetic_weights(cfg, int(case["seed"]))
    prompt = prompt[:len(case["prompt"])]
    assert np.array_equal(prompt, case["prompt"])
    assert _digest(w, cfg) == json.loads(str(case["weights_sha256"]))
    toks, logits = llama.LlamaOracle(cfg, w).generate(prompt, len(case["tokens"]), keep_logits=True)
    assert toks == [int(t) for t in case["tokens"]]
    from ml_dtypes import bfloat16
    got = np.stack([lg.astype(bfloat16).view(np.uint16) for lg in logits])
    assert np.array_equal(got, case["logits_bf16"])
