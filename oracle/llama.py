"""CPU oracle of the Llama-3.2 greedy decode path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's Llama CPU path (``use_npu=False``) for
BASELINE config 3 (Llama-3.2-1B shape, random-init Q4 weights):

* RoPE table with Llama-3 frequency scaling      runtime/py/model.py:230-261
* RMSNorm, eps 1e-5, times the norm weight        runtime/py/model.py:531-532
* half-split rotary embedding on bf16 q / k       runtime/py/model.py:534-550
* GQA attention over the bf16 KV cache            runtime/py/model.py:580-630
* the layer (QKV, RoPE, cache, attention, O, residual, RMSNorm, SwiGLU FFN,
  residual) with every ``.astype(bfloat16)``    runtime/py/model.py:821-864
* forward: embedding, 16 layers, final norm, LM head (the quantized tied
  embedding), bf16 logits                          runtime/py/model.py:919-934
* greedy generation: the prompt token by token without logits, then argmax
  (first index of the maximum)                     tests/test_generation.py:72-99
* the on-disk shapes of the quantized model: K and V padded to 2048 rows,
  the LM head padded to 129024 rows               tools/quantize_model.py:61-118

Only ``tests/`` and the golden-fixture scripts import it; the product path
never does.  The operations are numpy calls of the same kind, shape and
order as the reference's, so in one container the two agree bit for bit
(``tests/golden/make_llama_golden.py`` checks that against the reference's
own ``LlamaNPUModel`` methods).
"""
from __future__ import annotations

import numpy as np
from ml_dtypes import bfloat16

from . import q4

PROJ = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


class Config:
    """Llama-3.2-1B decode shape (the reference's defaults, model.py:94-101)."""

    def __init__(self, hidden=2048, intermediate=8192, heads=32, kv_heads=8, head_dim=64, layers=16,
                 vocab=128256, vocab_padded=129024, max_seq=512, rope_theta=500000.0):
        self.hidden, self.intermediate = hidden, intermediate
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.layers, self.vocab, self.vocab_padded = layers, vocab, vocab_padded
        self.max_seq, self.rope_theta = max_seq, rope_theta

    def shapes(self) -> dict:
        """On-disk (rows, cols) of each packed matrix (tools/quantize_model.py:85-118:
        K and V padded to `hidden` rows)."""
        H, I = self.hidden, self.intermediate
        kvp = max(H, self.kv_heads * self.head_dim)
        return {"attn_q": (H, H), "attn_k": (kvp, H), "attn_v": (kvp, H), "attn_output": (H, H),
                "ffn_gate": (I, H), "ffn_up": (I, H), "ffn_down": (H, I)}


def synthetic_weights(cfg: Config, seed: int = 0, quantize=None):
    """Random-init Q4 model of BASELINE config 3: every matrix
    N(0, 0.02) in float32 (numpy ``default_rng(seed).standard_normal(...,
    float32) * 0.02``), quantized with `quantize` (default: the oracle's
    restatement of quantize_to_q4_0 + pack_to_combined); K and V rows beyond
    kv_heads*head_dim are zero (the padding of tools/quantize_model.py); norm
    weights 1; token_embd N(0, 0.02) as float16; the LM head is the quantized
    float32 embedding padded to vocab_padded rows (quantize_model.py:61-70).
    Also returns the prompt: 128 ids ``integers(0, vocab)`` of a second
    generator seeded seed + 1.

    Generation order (fixed): token_embd, then per layer the projections in
    PROJ order."""
    quantize = quantize or q4.quantize_combined
    rng = np.random.default_rng(seed)
    H = cfg.hidden
    emb = (rng.standard_normal((cfg.vocab, H), dtype=np.float32) * np.float32(0.02)).astype(np.float16)
    w = {"token_embd": emb, "output_norm.weight": np.ones(H, np.float32)}
    lm = np.zeros((cfg.vocab_padded, H), np.float32)
    lm[:cfg.vocab] = emb.astype(np.float32)
    w["lm_head_packed"] = quantize(lm)
    del lm
    kv = cfg.kv_heads * cfg.head_dim
    for l in range(cfg.layers):
        w[f"blk.{l}.attn_norm.weight"] = np.ones(H, np.float32)
        w[f"blk.{l}.ffn_norm.weight"] = np.ones(H, np.float32)
        for proj in PROJ:
            rows, cols = cfg.shapes()[proj]
            real = kv if proj in ("attn_k", "attn_v") else rows
            m = np.zeros((rows, cols), np.float32)
            m[:real] = rng.standard_normal((real, cols), dtype=np.float32) * np.float32(0.02)
            w[f"blk.{l}.{proj}.weight_packed"] = quantize(m)
            del m
    prompt = np.random.default_rng(seed + 1).integers(0, cfg.vocab, 128).astype(np.int64)
    return w, prompt


def rope_table(cfg: Config) -> np.ndarray:
    """cos/sin table, bf16 (max_seq, 2*head_dim): [cos, cos, sin, sin] per
    position with Llama-3 frequency scaling (factor 32, low 1, high 4, old
    context 8192).  Restates runtime/py/model.py:230-261."""
    dim = cfg.head_dim
    base, factor, low_ff, high_ff, old_ctx = cfg.rope_theta, 32.0, 1.0, 4.0, 8192
    inv_freq = 1.0 / (base ** (np.arange(0, dim, 2, dtype=np.float32) / dim))
    low_wl = old_ctx / low_ff
    high_wl = old_ctx / high_ff
    wavelen = 2 * np.pi / inv_freq
    inv_l = inv_freq.copy()
    inv_l = np.where(wavelen > low_wl, inv_freq / factor, inv_l)
    smooth = (old_ctx / wavelen - low_ff) / (high_ff - low_ff)
    smooth = np.clip(smooth, 0.0, 1.0)
    smoothed = (1 - smooth) * (inv_freq / factor) + smooth * inv_freq
    medium = (wavelen >= high_wl) & (wavelen <= low_wl)
    inv_l = np.where(medium, smoothed, inv_l)
    table = np.zeros((cfg.max_seq, 2 * dim), dtype=np.float32)
    for pos in range(cfg.max_seq):
        freqs = pos * inv_l
        c, s = np.cos(freqs), np.sin(freqs)
        table[pos] = np.concatenate([np.concatenate([c, c]), np.concatenate([s, s])])
    return table.astype(bfloat16)


def rmsnorm(x_bf, w):
    """runtime/py/model.py:531-532 (Llama branch)."""
    variance = np.mean(x_bf.astype(np.float32) ** 2)
    return (x_bf.astype(np.float32) * (1.0 / np.sqrt(variance + 1e-5)) * w).astype(bfloat16)


def rope(x_bf, pos, table, head_dim=64):
    """runtime/py/model.py:534-550."""
    half = head_dim // 2
    cs = table[pos]
    cos = cs[:half].astype(np.float32)
    sin = cs[head_dim:head_dim + half].astype(np.float32)
    nh = x_bf.shape[0] // head_dim
    x = x_bf.astype(np.float32).reshape(nh, head_dim)
    y = np.zeros_like(x)
    for h in range(nh):
        x1 = x[h, :half]
        x2 = x[h, half:]
        y[h, :half] = x1 * cos - x2 * sin
        y[h, half:] = x2 * cos + x1 * sin
    return y.reshape(-1).astype(bfloat16)


class LlamaOracle:
    """The reference's Llama CPU decode path on a weight dict as written by
    synthetic_weights (or read from a quantized-model directory)."""

    def __init__(self, cfg: Config, weights: dict):
        self.cfg = cfg
        self.emb = weights["token_embd"]
        self.out_norm = weights["output_norm.weight"]
        self.attn_norm = [weights[f"blk.{l}.attn_norm.weight"] for l in range(cfg.layers)]
        self.ffn_norm = [weights[f"blk.{l}.ffn_norm.weight"] for l in range(cfg.layers)]
        # bf16-valued float32 copies of the dequantized matrices (the
        # reference keeps bf16 copies and widens them on every call,
        # model.py:135-145; the values are the same)
        self.W = [{p: q4.dequantize_combined(weights[f"blk.{l}.{p}.weight_packed"]) for p in PROJ}
                  for l in range(cfg.layers)]
        self.lm = q4.dequantize_combined(weights["lm_head_packed"])
        self.table = rope_table(cfg)
        shape = (cfg.kv_heads, cfg.max_seq, cfg.head_dim)
        self.k_cache = [np.zeros(shape, dtype=bfloat16) for _ in range(cfg.layers)]
        self.v_cache = [np.zeros(shape, dtype=bfloat16) for _ in range(cfg.layers)]

    def reset(self):
        for c in self.k_cache + self.v_cache:
            c.fill(0)

    def attention(self, q_rope, pos, l):
        """runtime/py/model.py:580-630 (no sliding window on Llama)."""
        cfg = self.cfg
        nh, nkv, dim = cfg.heads, cfg.kv_heads, cfg.head_dim
        scale = 1.0 / np.sqrt(dim)
        q = q_rope.astype(np.float32).reshape(nh, dim)
        seq_len = pos + 1
        k = self.k_cache[l][:, :seq_len, :].astype(np.float32)
        v = self.v_cache[l][:, :seq_len, :].astype(np.float32)
        g = nh // nkv
        if g > 1:
            k = np.repeat(k, g, axis=0)
            v = np.repeat(v, g, axis=0)
        scores = np.zeros((nh, seq_len), dtype=np.float32)
        for h in range(nh):
            scores[h] = np.dot(k[h], q[h]) * scale
        mx = np.max(scores, axis=-1, keepdims=True)
        e = np.exp(scores - mx)
        probs = e / np.sum(e, axis=-1, keepdims=True)
        out = np.zeros((nh, dim), dtype=np.float32)
        for h in range(nh):
            out[h] = np.dot(probs[h], v[h])
        return out.reshape(-1).astype(bfloat16)

    def layer(self, x, pos, l):
        """runtime/py/model.py:821-864 (use_npu=False)."""
        cfg = self.cfg
        W = self.W[l]
        kv = cfg.kv_heads * cfg.head_dim
        xn = rmsnorm(x, self.attn_norm[l])
        q = (W["attn_q"] @ xn.astype(np.float32)).astype(bfloat16)
        k = (W["attn_k"] @ xn.astype(np.float32)).astype(bfloat16)[:kv]
        v = (W["attn_v"] @ xn.astype(np.float32)).astype(bfloat16)[:kv]
        q_rope = rope(q, pos, self.table, cfg.head_dim)
        k_rope = rope(k, pos, self.table, cfg.head_dim)
        self.k_cache[l][:, pos, :] = k_rope.reshape(cfg.kv_heads, cfg.head_dim)
        self.v_cache[l][:, pos, :] = v.reshape(cfg.kv_heads, cfg.head_dim)
        attn = self.attention(q_rope, pos, l)
        proj = (W["attn_output"] @ attn.astype(np.float32)).astype(bfloat16)
        x_post = (x.astype(np.float32) + proj.astype(np.float32)).astype(bfloat16)
        xn2 = rmsnorm(x_post, self.ffn_norm[l])
        gate = (W["ffn_gate"] @ xn2.astype(np.float32)).astype(bfloat16)
        up = (W["ffn_up"] @ xn2.astype(np.float32)).astype(bfloat16)
        g32 = gate.astype(np.float32)
        u32 = up.astype(np.float32)
        act = ((g32 * (1.0 / (1.0 + np.exp(-g32)))) * u32).astype(bfloat16)
        down = (W["ffn_down"] @ act.astype(np.float32)).astype(bfloat16)
        return (x_post.astype(np.float32) + down.astype(np.float32)).astype(bfloat16)

    def forward(self, token: int, pos: int, return_logits: bool = True):
        """runtime/py/model.py:919-934; bf16 logits widened to float32."""
        x = self.emb[token].astype(bfloat16)
        for l in range(self.cfg.layers):
            x = self.layer(x, pos, l)
        if not return_logits:
            return None
        xn = rmsnorm(x, self.out_norm)
        logits = (self.lm @ xn.astype(np.float32)).astype(bfloat16)
        return logits[:self.cfg.vocab].astype(np.float32)

    def generate(self, prompt, steps: int, keep_logits: bool = False):
        """Greedy decode (tests/test_generation.py:72-99 without the EOS
        stop): the prompt token by token, then `steps` argmax tokens."""
        self.reset()
        for pos in range(len(prompt) - 1):
            self.forward(int(prompt[pos]), pos, return_logits=False)
        tok, pos = int(prompt[-1]), len(prompt) - 1
        out, logits = [], []
        for _ in range(steps):
            lg = self.forward(tok, pos)
            tok = int(np.argmax(lg))
            out.append(tok)
            if keep_logits:
                logits.append(lg)
            pos += 1
        return (out, logits) if keep_logits else out


def top2_gap(logits: np.ndarray) -> tuple[int, float, float]:
    """(argmax, max, the largest value at another index): the margin by which
    the greedy choice wins (0 for a tie broken by the lower index)."""
    i = int(np.argmax(logits))
    m = float(logits[i])
    rest = np.delete(logits, i)
    return i, m, float(rest.max())
