"""The producer side of the on-disk format (alveare_b200.quantize, restating
tools/quantize_model.py:12-125) on a tiny Llama-shaped model, with the
oracle's quantizer plugged in (the GPU quantizer is bit-exact with it,
tests/test_gemv_gpu.py): file names, dtypes, padding rows and the RoPE
un-permutation."""
import json

import numpy as np

from alveare_b200.quantize import quantize_llama, unpermute
from oracle import q4


def llama_cpp_permute(w, n_head):
    """llama.cpp's conversion permutation of Q / K rows (the inverse of unpermute)."""
    return w.reshape(n_head, 2, w.shape[0] // n_head // 2, *w.shape[1:]).swapaxes(1, 2).reshape(w.shape)


def test_unpermute_inverts_llama_cpp_permutation():
    w = np.random.default_rng(0).normal(size=(256, 64)).astype(np.float32)
    for heads in (2, 4, 8):
        assert np.array_equal(unpermute(llama_cpp_permute(w, heads), heads), w)


def test_quantize_llama_directory(tmp_path):
    rng = np.random.default_rng(1)
    H, I, V, heads, kv, L = 64, 128, 100, 2, 1, 2
    hd = H // heads
    t = {"token_embd.weight": rng.normal(0, 0.02, (V, H)).astype(np.float32),
         "output_norm.weight": np.ones(H, np.float32)}
    shapes = {"attn_q": (H, H), "attn_k": (kv * hd, H), "attn_v": (kv * hd, H), "attn_output": (H, H),
              "ffn_gate": (I, H), "ffn_up": (I, H), "ffn_down": (H, I)}
    for l in range(L):
        t[f"blk.{l}.attn_norm.weight"] = np.ones(H, np.float32)
        t[f"blk.{l}.ffn_norm.weight"] = np.ones(H, np.float32)
        for p, s in shapes.items():
            t[f"blk.{l}.{p}.weight"] = rng.normal(0, 0.02, s).astype(np.float32)
    cfg = quantize_llama(t, tmp_path, heads=heads, kv_heads=kv, quantize=q4.quantize_combined)
    assert cfg["num_hidden_layers"] == L and cfg["vocab_size"] == V and cfg["head_dim"] == hd
    assert json.load(open(tmp_path / "config.json")) == cfg
    emb = np.load(tmp_path / "token_embd.npy")
    assert emb.dtype == np.float16 and emb.shape == (V, H)
    lm = np.load(tmp_path / "lm_head_packed.npy")
    assert lm.shape == (2048, H // 32 * 20)                      # vocabulary padded to 2048 rows
    deq = q4.dequantize_combined(lm)
    assert np.array_equal(deq[V:], np.zeros_like(deq[V:]))       # padding rows dequantize to zero
    for l in range(L):
        qk = np.load(tmp_path / f"blk.{l}.attn_q.weight_packed.npy")
        assert np.array_equal(qk, q4.quantize_combined(unpermute(t[f"blk.{l}.attn_q.weight"], heads)))
        kk = np.load(tmp_path / f"blk.{l}.attn_k.weight_packed.npy")
        assert kk.shape == (H, H // 32 * 20)                     # K padded to `hidden` rows
        assert np.array_equal(kk[:kv * hd], q4.quantize_combined(unpermute(t[f"blk.{l}.attn_k.weight"], kv)))
        vv = np.load(tmp_path / f"blk.{l}.attn_v.weight_packed.npy")
        assert np.array_equal(vv[:kv * hd], q4.quantize_combined(t[f"blk.{l}.attn_v.weight"]))
        dn = np.load(tmp_path / f"blk.{l}.ffn_down.weight_packed.npy")
        assert dn.shape == (H, I // 32 * 20)
        assert np.load(tmp_path / f"blk.{l}.ffn_norm.weight.npy").dtype == np.float32
