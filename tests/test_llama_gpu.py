"""Llama greedy decode on the GPU (alv_llama_*, alveare_b200.llama) against
the CPU oracle (oracle/llama.py: the reference's use_npu=False path,
runtime/py/model.py:821-934) and against the greedy tokens the reference's
own code produced for BASELINE config 3 (tests/golden/llama_config3.json,
written by tests/golden/make_llama_golden.py).

Numerics: every rounding point of the reference is reproduced (bf16 after
each projection, norm, RoPE, attention and residual; fp32 inside), but fp32
sums run in another order than numpy's, so an occasional bf16 rounding of a
hidden state flips.  Logits are therefore held to a normwise bound per step
(teacher-forced: both sides consume the same tokens), greedy tokens must
match wherever the reference's top-two logits are apart (bf16 logits tie
exactly now and then, and a tie is decided by the last bit of an fp32 sum)."""
import hashlib
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from alveare_b200 import q4_quantize  # noqa: E402
from alveare_b200.llama import LlamaConfig, LlamaDecoder  # noqa: E402
from oracle import llama, q4  # noqa: E402

LOGIT_TOL = 2e-2   # normwise, bf16 logits after a teacher-forced step


def gpu_quantize(W):
    """quantize_to_q4_0 + pack_to_combined on the GPU (bit-exact with the
    reference's quantizer, tests/test_gemv_gpu.py); host result."""
    return q4_quantize(torch.from_numpy(np.ascontiguousarray(W)).cuda()).cpu().numpy()


def small_config():
    return llama.Config(hidden=256, intermediate=512, heads=4, kv_heads=2, head_dim=64, layers=2, vocab=1000,
                        vocab_padded=1024, max_seq=64)


def decoder_for(cfg, w, per_kernel_step=0):
    c = LlamaConfig(cfg.hidden, cfg.intermediate, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.layers, cfg.vocab,
                    cfg.max_seq, 1e-5, per_kernel_step)
    return LlamaDecoder(w, c, device=0, rope_theta=cfg.rope_theta)


def normwise(y, ref):
    return float(np.max(np.abs(np.asarray(y, np.float64) - ref)) / np.max(np.abs(ref)))


def test_rope_table_matches_oracle():
    from alveare_b200.llama import rope_table
    cfg = llama.Config(max_seq=300)
    assert np.array_equal(rope_table(64, 300), llama.rope_table(cfg).view(np.uint16))


def test_small_model_forward_and_generate_against_oracle():
    cfg = small_config()
    w, _ = llama.synthetic_weights(cfg, seed=3)
    prompt = [5, 17, 999, 0, 42, 7, 7, 300]
    orc = llama.LlamaOracle(cfg, w)
    dec = decoder_for(cfg, w)
    # teacher-forced forwards: the same token stream into both
    ref_toks, ref_logits = orc.generate(prompt, 12, keep_logits=True)
    stream = prompt + ref_toks
    dec.reset_caches()
    for pos in range(len(prompt) - 1):
        assert dec.forward(stream[pos], pos, return_logits=False) is None
    for s in range(12):
        pos = len(prompt) - 1 + s
        lg = dec.forward(stream[pos], pos)
        ref = ref_logits[s]
        assert normwise(lg, ref) <= LOGIT_TOL
        i, mx, second = llama.top2_gap(ref)
        if mx - second > 2 * 2.0 ** (np.floor(np.log2(abs(mx))) - 7):   # more than two bf16 steps apart
            assert int(np.argmax(lg)) == i
    # the device-side greedy loop (graphs) against the oracle's greedy tokens
    got = dec.generate(prompt, 12)
    agree = next((k for k, (a, b) in enumerate(zip(got, ref_toks)) if a != b), len(got))
    assert agree >= 8, (got, ref_toks)
    # twice: the graphs are replayed, the cache is reset by generate
    assert dec.generate(prompt, 12) == got
    # steps that would consume position max_seq are refused before any launch
    from alveare_b200._lib import AlvError
    dec.start(prompt)
    with pytest.raises(AlvError):
        dec.run(len(prompt), cfg.max_seq - len(prompt) + 1)
    dec.run(len(prompt) - 1, cfg.max_seq - len(prompt) - 1)
    with pytest.raises(AlvError):
        dec.run(0, 3)
    dec.run(0, 2)   # positions max_seq - 2 and max_seq - 1
    with pytest.raises(AlvError):
        dec.prefill(cfg.max_seq - 3, 4)
    dec.prefill(0, 4)
    dec.run(0, cfg.max_seq - 4)
    with pytest.raises(AlvError):
        dec.run(1, 0)
    assert dec.generate(prompt, 12) == got
    dec.free()


def test_one_launch_step_equals_separate_kernels():
    """The one-launch step (llama_step_kernel: every layer, the LM head and
    the argmax in one persistent kernel) computes exactly what the
    separate-kernel step computes: bit-identical logits at every position
    and the same greedy tokens.  The small model's projections exercise the
    unit-balanced partitions (rows split between CTAs) as well as the
    row-aligned ones."""
    cfg = small_config()
    w, _ = llama.synthetic_weights(cfg, seed=11)
    one = decoder_for(cfg, w)
    sep = decoder_for(cfg, w, per_kernel_step=1)
    assert one.one_launch() and not sep.one_launch()
    stream = [3, 999, 17, 17, 0, 512, 64, 5, 900, 1, 2, 3]
    one.reset_caches()
    sep.reset_caches()
    for pos, tok in enumerate(stream):
        a = one.forward(tok, pos)
        b = sep.forward(tok, pos)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), pos
    prompt = [5, 17, 999, 0, 42]
    assert one.generate(prompt, 20) == sep.generate(prompt, 20)
    one.free()
    sep.free()


def test_batched_prefill_matches_token_by_token():
    """Batched prefill (tcgen05 gemms over the prompt rows, causal attention
    per row) fills the KV cache as the token-by-token path does: the logits
    of the step after the prompt agree normwise (the gemm sums in another
    order than the gemv, so bf16 values differ in their last bits), the
    greedy continuation follows the oracle's, and a prompt longer than one
    batch of 256 rows is handled in pieces."""
    cfg = small_config()
    cfg.max_seq = 600
    w, _ = llama.synthetic_weights(cfg, seed=4)
    dec = decoder_for(cfg, w)
    rng = np.random.default_rng(9)
    for n_prompt in (9, 300):
        prompt = [int(t) for t in rng.integers(0, cfg.vocab, n_prompt)]
        dec.start(prompt)
        dec.run(n_prompt - 1, 0)
        ref = dec.forward(prompt[-1], n_prompt - 1)
        dec.start(prompt)
        dec.prefill(0, n_prompt - 1)
        got = dec.forward(prompt[-1], n_prompt - 1)
        assert normwise(got, ref) <= LOGIT_TOL, n_prompt
        assert int(np.argmax(got)) == int(np.argmax(ref))
    prompt = [5, 17, 999, 0, 42, 7, 7, 300]
    orc = llama.LlamaOracle(cfg, w)
    ref_toks = orc.generate(prompt, 12)
    got = dec.generate(prompt, 12, batch_prefill=True)
    agree = next((k for k, (a, b) in enumerate(zip(got, ref_toks)) if a != b), len(got))
    assert agree >= 8, (got, ref_toks)
    dec.free()


GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "llama_config3.json")


def bf16_ulp(v: float) -> float:
    return 2.0 ** (np.floor(np.log2(abs(v))) - 7)


def near_tie(step: dict, ulps: float = 4.0) -> bool:
    """The reference's greedy choice wins by at most `ulps` bf16 steps (0 is
    an exact tie of bf16 logits, broken by the lower index)."""
    return step["max"] - step["second"] <= ulps * bf16_ulp(step["max"])


@pytest.mark.skipif(not os.path.exists(GOLDEN), reason="config-3 golden tokens not generated")
def test_config3_greedy_tokens_match_reference():
    """Llama-3.2-1B shape, random-init Q4 (seed 0), a
    128-token random prompt and 256 greedy steps.  The weights are rebuilt
    here (the GPU quantizer is bit-exact with the reference's, checked by
    the sha256 digests) and the GPU's tokens compared with the reference's.

    The logits are bf16, so the reference meets exact ties (step 11 of this
    run: two tokens at 3.875, the lower index wins); there a one-ulp
    difference in an fp32 sum decides, and no different-order fp32
    arithmetic can promise the same pick.  The GPU's fp32 sums (tensor-core
    accumulation, another order) differ from numpy's in the last bits, which
    flips some of the ~700,000 bf16 roundings of a decode step; over 16
    layers and the KV cache the bf16 logits drift by up to a few bf16 steps
    (measured: up to 6 steps, most within 1).  So: free-running, the GPU must
    follow the reference up to a step where the reference's top two logits
    are within four bf16 steps; teacher-forced on the reference's sequence,
    every step with a clear margin must pick the reference's token, and at
    most 1 in 8 steps may differ."""
    gold = json.load(open(GOLDEN))
    cfg = llama.Config(max_seq=512)
    w, prompt = llama.synthetic_weights(cfg, seed=gold["seed"], quantize=gpu_quantize)
    assert [int(t) for t in prompt] == gold["prompt"]
    assert hashlib.sha256(w["lm_head_packed"].tobytes()).hexdigest() == gold["weights_sha256"]["lm_head_packed"]
    hsh = hashlib.sha256()
    for l in range(cfg.layers):
        for p in llama.PROJ:
            hsh.update(w[f"blk.{l}.{p}.weight_packed"].tobytes())
    assert hsh.hexdigest() == gold["weights_sha256"]["layers_packed"]
    dec = decoder_for(cfg, w)
    del w
    ref = gold["tokens"]
    steps = len(ref)
    got = dec.generate(gold["prompt"], steps)
    agree = next((k for k, (a, b) in enumerate(zip(got, ref)) if a != b), steps)
    print(f"config 3: free-running GPU greedy tokens equal the reference's for {agree} of {steps} steps")
    if agree < steps:
        assert near_tie(gold["steps"][agree]), gold["steps"][agree]
    forced = dec.teacher_forced(gold["prompt"] + ref, len(gold["prompt"]))
    miss = [k for k in range(steps) if forced[k] != ref[k]]
    print(f"config 3: teacher-forced, {steps - len(miss)} of {steps} steps pick the reference's token; "
          f"the others are near ties: {[(k, gold['steps'][k]['max'], gold['steps'][k]['second']) for k in miss]}")
    assert all(near_tie(gold["steps"][k]) for k in miss)
    # how many near ties flip depends on the fp32 summation order (the
    # kernels' warps per CTA): 15 with 15 warps, 18 with 16
    assert len(miss) <= steps // 8
    # batched prefill of the prompt: the same criterion as free-running
    got_b = dec.generate(gold["prompt"], steps, batch_prefill=True)
    agree_b = next((k for k, (a, b) in enumerate(zip(got_b, ref)) if a != b), steps)
    print(f"config 3: with batched prefill, greedy tokens equal the reference's for {agree_b} of {steps} steps")
    if agree_b < steps:
        assert near_tie(gold["steps"][agree_b]), gold["steps"][agree_b]
    # the separate-kernel step predicts exactly the same tokens
    if dec.one_launch():
        sep = decoder_for(cfg, llama.synthetic_weights(cfg, seed=gold["seed"], quantize=gpu_quantize)[0],
                          per_kernel_step=1)
        assert sep.teacher_forced(gold["prompt"] + ref, len(gold["prompt"])) == forced
        assert sep.generate(gold["prompt"], steps) == got
        sep.free()
    dec.free()


def test_quantized_directory_round_trip(tmp_path):
    """Float weights -> the reference's quantized-model directory on the GPU
    (alveare_b200.quantize, tools/quantize_model.py) -> LlamaDecoder(dir):
    the same greedy tokens as the oracle reading that directory."""
    from alveare_b200.llama import load_weights_dir
    from alveare_b200.quantize import quantize_llama
    rng = np.random.default_rng(5)
    H, I, V, heads, kv, L = 256, 512, 1000, 4, 2, 2
    hd = H // heads
    t = {"token_embd.weight": rng.normal(0, 0.02, (V, H)).astype(np.float32), "output_norm.weight": np.ones(H, np.float32)}
    shapes = {"attn_q": (H, H), "attn_k": (kv * hd, H), "attn_v": (kv * hd, H), "attn_output": (H, H),
              "ffn_gate": (I, H), "ffn_up": (I, H), "ffn_down": (H, I)}
    for l in range(L):
        t[f"blk.{l}.attn_norm.weight"] = np.ones(H, np.float32)
        t[f"blk.{l}.ffn_norm.weight"] = np.ones(H, np.float32)
        for p, s in shapes.items():
            t[f"blk.{l}.{p}.weight"] = rng.normal(0, 0.02, s).astype(np.float32)
    quantize_llama(t, tmp_path, heads=heads, kv_heads=kv)
    w = load_weights_dir(tmp_path, L)
    assert np.array_equal(w["blk.1.ffn_up.weight_packed"], q4.quantize_combined(t["blk.1.ffn_up.weight"]))
    cfg = llama.Config(hidden=H, intermediate=I, heads=heads, kv_heads=kv, head_dim=hd, layers=L, vocab=V,
                       vocab_padded=2048, max_seq=2048)
    orc = llama.LlamaOracle(cfg, {k: np.asarray(v) for k, v in w.items()})
    prompt = [1, 2, 3, 500, 999]
    ref = orc.generate(prompt, 6)
    dec = LlamaDecoder(str(tmp_path))
    assert dec.cfg.hidden == H and dec.cfg.layers == L
    got = dec.generate(prompt, 6)
    agree = next((k for k, (a, b) in enumerate(zip(got, ref)) if a != b), len(got))
    assert agree >= 4, (got, ref)
    dec.free()
