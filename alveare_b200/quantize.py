"""Producer side of the on-disk Q4 model format: float weights -> the
reference's quantized-model directory, which :class:`alveare_b200.llama.LlamaDecoder`
(and the reference's own runtime, runtime/py/model.py:38-127) loads.

Restates tools/quantize_model.py:12-125 for a Llama-style model given as
float arrays by their GGUF tensor names:

* ``token_embd.npy``          the embedding as float16 (the host-side lookup, :61-64)
* ``lm_head_packed.npy``      the tied LM head: the embedding in float32,
                              vocabulary rows zero-padded to a multiple of 2048
                              (128256 -> 129024), quantized and packed (:66-70)
* ``*norm.weight.npy``        norm weights as float32 (:73-76)
* ``blk.{l}.attn_q / attn_k.weight_packed.npy``  Q and K un-permuted from
                              llama.cpp's RoPE layout (:25-30, :78-92); K (and V,
                              :101-106) zero-padded to `hidden` rows
* the other projections       quantized and packed as they are (:94-118)
* ``config.json``             the shapes (read back by LlamaDecoder)

Quantization is the reference's Q4_0 (tools/convert/gemv_q_convert.py:5-85)
done on the GPU by ``alv_q4_quantize`` (bit-exact with the reference's numpy
quantizer); a different ``quantize`` callable may be passed.  Reading GGUF
files is left to the caller (the tensors only need to be arrays).
"""
from __future__ import annotations

import json
import os

import numpy as np

PROJ = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


def unpermute(weights: np.ndarray, n_head: int) -> np.ndarray:
    """Undo llama.cpp's RoPE row permutation of a Q or K projection: rows of
    each head go from interleaved (pairs) back to the half-split order the
    decode path rotates (tools/quantize_model.py:22-27)."""
    head_dim = weights.shape[0] // n_head
    return (weights.reshape(n_head, head_dim // 2, 2, weights.shape[1]).swapaxes(1, 2)
            .reshape(weights.shape))


def pad_rows(W: np.ndarray, rows: int) -> np.ndarray:
    """Zero rows appended up to `rows` (tools/quantize_model.py:12-20)."""
    if W.shape[0] >= rows:
        return W
    out = np.zeros((rows, W.shape[1]), dtype=W.dtype)
    out[:W.shape[0]] = W
    return out


def gpu_quantize(W: np.ndarray, device: int = 0) -> np.ndarray:
    """quantize_to_q4_0 + pack_to_combined on the GPU; host result."""
    import torch

    from .ops import q4_quantize
    t = torch.from_numpy(np.ascontiguousarray(W, dtype=np.float32)).to(torch.device("cuda", device))
    return q4_quantize(t).cpu().numpy()


def quantize_llama(tensors: dict, out_dir, heads: int, kv_heads: int, rope_theta: float = 500000.0,
                   permuted: bool = True, quantize=None, device: int = 0) -> dict:
    """Write the quantized-model directory of a Llama-style model.

    tensors: float arrays by GGUF name (``token_embd.weight``,
    ``output_norm.weight``, ``blk.{l}.{attn_norm,ffn_norm}.weight`` and
    ``blk.{l}.{proj}.weight`` for the seven projections, each (out, in)).
    permuted: Q and K are in llama.cpp's RoPE layout (as GGUF stores them).
    Returns the config written to ``config.json``."""
    quantize = quantize or (lambda W: gpu_quantize(W, device))
    os.makedirs(out_dir, exist_ok=True)
    emb = np.asarray(tensors["token_embd.weight"])
    vocab, hidden = emb.shape
    np.save(os.path.join(out_dir, "token_embd.npy"), emb.astype(np.float16))
    vocab_padded = (vocab + 2047) // 2048 * 2048
    np.save(os.path.join(out_dir, "lm_head_packed.npy"), quantize(pad_rows(emb.astype(np.float32), vocab_padded)))
    np.save(os.path.join(out_dir, "output_norm.weight.npy"), np.asarray(tensors["output_norm.weight"], np.float32))
    layers = 0
    while f"blk.{layers}.attn_q.weight" in tensors:
        layers += 1
    intermediate = np.asarray(tensors["blk.0.ffn_gate.weight"]).shape[0] if layers else 0
    for l in range(layers):
        for norm in ("attn_norm", "ffn_norm"):
            np.save(os.path.join(out_dir, f"blk.{l}.{norm}.weight.npy"),
                    np.asarray(tensors[f"blk.{l}.{norm}.weight"], np.float32))
        for proj in PROJ:
            W = np.asarray(tensors[f"blk.{l}.{proj}.weight"], np.float32)
            if permuted and proj == "attn_q":
                W = unpermute(W, heads)
            if permuted and proj == "attn_k":
                W = unpermute(W, kv_heads)
            if proj in ("attn_k", "attn_v"):
                W = pad_rows(W, hidden)
            np.save(os.path.join(out_dir, f"blk.{l}.{proj}.weight_packed.npy"), quantize(W))
    cfg = {"model_type": "llama", "hidden_size": int(hidden), "intermediate_size": int(intermediate),
           "num_attention_heads": int(heads), "num_key_value_heads": int(kv_heads),
           "head_dim": int(hidden // heads), "num_hidden_layers": layers, "vocab_size": int(vocab),
           "rope_theta": float(rope_theta)}
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)
    return cfg
