"""Llama-3.2 greedy decode on the GPU, behind the reference model's interface.

The reference's ``LlamaNPUModel`` (runtime/py/model.py) runs the decode step
in numpy on the host and sends the Q4 matmuls to the NPU; its C++ runtime
does the same with a greedy ``Generator`` (runtime/cpp/src/generator.cpp:
15-52).  :class:`LlamaDecoder` keeps the model's public surface --
``forward(token_id, pos, return_logits)``, ``reset_caches()`` and a greedy
``generate`` -- and runs every stage on the GPU through the C ABI
(``alv_llama_*``): the Q4 matmuls on the library's streaming kernels, the
RMSNorm / RoPE / KV cache / attention / residual / argmax glue in its own
kernels, one CUDA graph per step with no host work per token.

Weights use the reference's quantized-model names (tools/quantize_model.py:
39-125): a directory of ``.npy`` files, or a dict of arrays with the same
names (numpy host arrays or torch CUDA tensors).  The KV cache is bf16, as
the reference's (runtime/py/model.py:173-174).
"""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np

from . import _lib

try:
    import torch
except Exception:  # pragma: no cover
    torch = None

PROJECTIONS = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


class LlamaConfig(ctypes.Structure):
    """alv_llama_config; defaults are Llama-3.2-1B (runtime/py/model.py:94-101)."""
    _fields_ = [("hidden", ctypes.c_int32), ("intermediate", ctypes.c_int32), ("heads", ctypes.c_int32),
                ("kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("layers", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("max_seq", ctypes.c_int32), ("rms_eps", ctypes.c_float),
                ("per_kernel_step", ctypes.c_int32), ("reserved", ctypes.c_int32 * 6)]

    @classmethod
    def llama32_1b(cls, max_seq: int = 2048, per_kernel_step: int = 0) -> "LlamaConfig":
        return cls(2048, 8192, 32, 8, 64, 16, 128256, max_seq, 1e-5, per_kernel_step)


def rope_table(head_dim: int, max_seq: int, theta: float = 500000.0) -> np.ndarray:
    """bf16 bit patterns (max_seq, 2*head_dim) of the reference's cos/sin table
    with Llama-3 frequency scaling (factor 32, low 1, high 4, original context
    8192), computed as runtime/py/model.py:230-261 computes it (float32
    numpy, then bf16)."""
    from ml_dtypes import bfloat16
    dim = head_dim
    factor, low_ff, high_ff, old_ctx = 32.0, 1.0, 4.0, 8192
    inv_freq = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float32) / dim))
    wavelen = 2 * np.pi / inv_freq
    low_wl, high_wl = old_ctx / low_ff, old_ctx / high_ff
    inv = np.where(wavelen > low_wl, inv_freq / factor, inv_freq.copy())
    smooth = np.clip((old_ctx / wavelen - low_ff) / (high_ff - low_ff), 0.0, 1.0)
    smoothed = (1 - smooth) * (inv_freq / factor) + smooth * inv_freq
    inv = np.where((wavelen >= high_wl) & (wavelen <= low_wl), smoothed, inv)
    table = np.zeros((max_seq, 2 * dim), dtype=np.float32)
    for pos in range(max_seq):
        f = pos * inv
        c, s = np.cos(f), np.sin(f)
        table[pos] = np.concatenate([c, c, s, s])
    return table.astype(bfloat16).view(np.uint16)


def load_weights_dir(weights_dir, layers: int) -> dict:
    """The tensors of a quantized-model directory by name (runtime/py/model.py:
    38-127 reads the same files)."""
    d = str(weights_dir)
    names = ["token_embd", "output_norm.weight", "lm_head_packed"]
    for l in range(layers):
        names += [f"blk.{l}.attn_norm.weight", f"blk.{l}.ffn_norm.weight"]
        names += [f"blk.{l}.{p}.weight_packed" for p in PROJECTIONS]
    return {n: np.load(os.path.join(d, n + ".npy"), mmap_mode="r") for n in names}


class LlamaDecoder:
    """Greedy Llama decode on one GPU (BASELINE config 3's model)."""

    def __init__(self, weights, config: LlamaConfig | None = None, device: int = 0, rope_theta: float = 500000.0):
        if not isinstance(weights, dict):
            cfg_path = os.path.join(str(weights), "config.json")
            if os.path.exists(cfg_path):
                c = json.load(open(cfg_path))
                rope_theta = float(c.get("rope_theta", rope_theta))
                if config is None and "hidden_size" in c:
                    config = LlamaConfig(c["hidden_size"], c["intermediate_size"], c["num_attention_heads"],
                                         c["num_key_value_heads"], c["head_dim"], c["num_hidden_layers"],
                                         c["vocab_size"], 2048, 1e-5)
        self.cfg = config or LlamaConfig.llama32_1b()
        self.device = device
        self.ctx = _lib.context(device)
        if not isinstance(weights, dict):
            weights = load_weights_dir(weights, self.cfg.layers)
        h = ctypes.c_uint32()
        self.ctx.check(self.ctx.lib.alv_llama_create(self.ctx.ptr, ctypes.byref(self.cfg), ctypes.byref(h)),
                       "alv_llama_create")
        self.handle = h.value
        for name, arr in weights.items():
            self._load(name, arr)
        self._load("rope_table", rope_table(self.cfg.head_dim, self.cfg.max_seq, rope_theta))
        self._logits = None

    def _load(self, name: str, arr) -> None:
        if torch is not None and isinstance(arr, torch.Tensor) and arr.is_cuda:
            t = arr.contiguous()
            rc = self.ctx.lib.alv_llama_load(self.ctx.ptr, self.handle, name.encode(), t.data_ptr(),
                                             t.numel() * t.element_size(), 1)
        else:
            a = np.ascontiguousarray(arr)
            rc = self.ctx.lib.alv_llama_load(self.ctx.ptr, self.handle, name.encode(), a.ctypes.data, a.nbytes, 0)
        self.ctx.check(rc, f"alv_llama_load({name})")

    def _stream(self):
        return torch.cuda.current_stream(self.device).cuda_stream if torch is not None else None

    # -- the reference model's surface ---------------------------------------
    def reset_caches(self) -> None:
        self.ctx.check(self.ctx.lib.alv_llama_reset(self.ctx.ptr, self.handle, self._stream()), "alv_llama_reset")

    def forward(self, token_id: int, pos: int, return_logits: bool = True):
        """One step (runtime/py/model.py:866-934): the token enters the KV
        cache at `pos`; returns the float32 logits (bf16 values) or None."""
        st = self._stream()
        if return_logits:
            if self._logits is None:
                self._logits = torch.empty(self.cfg.vocab, dtype=torch.int16, device=f"cuda:{self.device}")
            ptr = self._logits.data_ptr()
        else:
            ptr = None
        self.ctx.check(self.ctx.lib.alv_llama_forward(self.ctx.ptr, self.handle, int(token_id), int(pos), ptr, st),
                       "alv_llama_forward")
        if not return_logits:
            return None
        bits = self._logits.cpu().numpy().view(np.uint16)
        self.ctx.sync_status(st)
        return (bits.astype(np.uint32) << 16).view(np.float32)

    def generate(self, prompt_ids, max_new_tokens: int, batch_prefill: bool = False) -> list[int]:
        """Greedy decode: the prompt token by token (or, with batch_prefill,
        all but its last token in batched prefill: tcgen05 gemms over up to 256
        positions at a time), then `max_new_tokens` argmax tokens
        (tests/test_generation.py:72-99 without an EOS stop)."""
        if batch_prefill:
            self.start(prompt_ids)
            self.prefill(0, len(prompt_ids) - 1)
            self.run(0, max_new_tokens)
            return self.tokens(len(prompt_ids), max_new_tokens)
        p = np.ascontiguousarray(np.asarray(prompt_ids, dtype=np.int32))
        out = np.empty(max_new_tokens, dtype=np.int32)
        self.ctx.check(self.ctx.lib.alv_llama_generate(self.ctx.ptr, self.handle, p.ctypes.data, len(p),
                                                       max_new_tokens, out.ctypes.data, self._stream()),
                       "alv_llama_generate")
        return [int(t) for t in out]

    # -- split form for timing ------------------------------------------------
    def start(self, prompt_ids) -> None:
        p = np.ascontiguousarray(np.asarray(prompt_ids, dtype=np.int32))
        self._n_prompt = len(p)
        self.ctx.check(self.ctx.lib.alv_llama_start(self.ctx.ptr, self.handle, p.ctypes.data, len(p), self._stream()),
                       "alv_llama_start")

    def prefill(self, pos0: int, n: int) -> None:
        """Positions [pos0, pos0 + n) of the started sequence through every
        layer in batches (the reference's run_layer_batch, model.cpp:422-571);
        the next step consumes position pos0 + n."""
        self.ctx.check(self.ctx.lib.alv_llama_prefill(self.ctx.ptr, self.handle, pos0, n, self._stream()),
                       "alv_llama_prefill")

    def run(self, prompt_steps: int, decode_steps: int) -> None:
        self.ctx.check(self.ctx.lib.alv_llama_run(self.ctx.ptr, self.handle, prompt_steps, decode_steps,
                                                  self._stream()), "alv_llama_run")

    def tokens(self, first: int, n: int) -> list[int]:
        out = np.empty(n, dtype=np.int32)
        self.ctx.check(self.ctx.lib.alv_llama_tokens(self.ctx.ptr, self.handle, first, n, out.ctypes.data,
                                                     self._stream()), "alv_llama_tokens")
        return [int(t) for t in out]

    def predicted(self, first: int, n: int) -> list[int]:
        """Argmax predictions for positions [first, first + n) (teacher-forced
        over a prompt, the greedy tokens past it)."""
        out = np.empty(n, dtype=np.int32)
        self.ctx.check(self.ctx.lib.alv_llama_predicted(self.ctx.ptr, self.handle, first, n, out.ctypes.data,
                                                        self._stream()), "alv_llama_predicted")
        return [int(t) for t in out]

    def teacher_forced(self, sequence, n_context: int) -> list[int]:
        """Feed `sequence` (context then continuation) and return the argmax
        predicted at every continuation position: the model's next-token
        choice given the true prefix, one greedy step per position."""
        self.start(sequence)
        self.run(n_context - 1, len(sequence) - n_context)
        return self.predicted(n_context, len(sequence) - n_context)

    def one_launch(self) -> bool:
        """Whether a step runs as one kernel launch (else separate kernels);
        known once the model is built (the first step builds it)."""
        info = (ctypes.c_int64 * 8)()
        self.ctx.check(self.ctx.lib.alv_llama_info(self.ctx.ptr, self.handle, info), "alv_llama_info")
        return bool(info[0])

    def free(self) -> None:
        if self.handle:
            self.ctx.lib.alv_weight_destroy(self.ctx.ptr, self.handle)
            self.handle = 0
