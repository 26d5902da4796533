"""Model-level wrappers of the reference's decode loop, on the B200.

The reference's ``LlamaNPUModel`` calls its NPU through three methods
(runtime/py/model.py:283-485):

* ``run_gemv_npu(W_combined, x_bf16) -> bf16 (N,)``    (:283-361)
* ``run_ffn_fused_npu(l, x_bf16) -> bf16 (H,)``         (:363-397)
* ``run_gemm_npu(W_combined, x_bf16 (B, K)) -> bf16 (B, N)``  (:399-485)

:class:`GpuModelOps` has the same three methods with the same arguments and
return values (host numpy arrays of ml_dtypes bfloat16), so a model object
can be switched by assigning them (``model.run_gemv_npu =
ops.run_gemv_npu`` ...) or by subclassing.  What changes underneath:

* Packed weights are repacked into the GPU unit layout once and kept
  resident, keyed by the packed array's identity (the reference re-uploads a
  non-resident matrix on every call, :291-295, 355-356); a :class:`Q4Weight`
  may be passed directly.
* No MAX_N / MAX_K chunking (:296-343) and no batch padding to 16
  (:415-478): one kernel call covers any N, K and B, and y is rounded to bf16
  once from the fp32 result, not per NPU chunk.
* The FFN returns the full down projection; the reference's host sum over
  per-core partials (:394-395) has one term.

``load_layer_weights`` reads the reference's on-disk layer files
(``blk.{l}.{proj}.weight_packed.npy``, runtime/py/model.py:38-52).
"""
from __future__ import annotations

import os

import numpy as np

from .ops import FusedFFNWeight, Q4Weight, _host_array

try:
    import torch
except Exception:  # pragma: no cover
    torch = None

PROJECTIONS = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")


def _bf16_type():
    from ml_dtypes import bfloat16
    return bfloat16


def load_layer_weights(weights_dir, layer: int) -> dict:
    """The packed (rows, cols/32*20) uint8 matrices of one layer that exist
    in `weights_dir`, by projection name (runtime/py/model.py:38-52)."""
    out = {}
    for proj in PROJECTIONS:
        path = os.path.join(str(weights_dir), f"blk.{layer}.{proj}.weight_packed.npy")
        if os.path.exists(path):
            out[proj] = np.load(path)
    return out


class GpuModelOps:
    """The reference model's three NPU entry points on one GPU."""

    def __init__(self, device: int = 0, activation: str = "silu"):
        if torch is None or not torch.cuda.is_available():
            raise RuntimeError("GpuModelOps needs a CUDA device")
        self.device = device
        self.activation = activation
        self._resident: dict[int, tuple[object, Q4Weight]] = {}
        self.layer_ffn: dict[int, FusedFFNWeight] = {}

    # -- weights ------------------------------------------------------------
    def resident(self, W_combined) -> Q4Weight:
        """The resident GPU copy of a packed matrix (repacked on first use)."""
        if isinstance(W_combined, Q4Weight):
            return W_combined
        key = id(W_combined)
        hit = self._resident.get(key)
        if hit is not None and hit[0] is W_combined:
            return hit[1]
        w = Q4Weight(W_combined, device=self.device)
        self._resident[key] = (W_combined, w)   # holding W keeps its id unique
        return w

    def register_ffn_layer(self, l: int, w_gate, w_up, w_down, H: int, I: int,
                           activation: str | None = None) -> FusedFFNWeight:
        """Make layer l's FFN resident (the reference's pack_ffn_fused_weights
        at load time, model.py:176-195)."""
        w = FusedFFNWeight(w_gate, w_up, w_down, H, I, activation or self.activation, device=self.device)
        old = self.layer_ffn.pop(l, None)
        if old is not None:
            old.free()
        self.layer_ffn[l] = w
        return w

    def free(self) -> None:
        for _, w in self._resident.values():
            w.free()
        self._resident.clear()
        for w in self.layer_ffn.values():
            w.free()
        self.layer_ffn.clear()

    # -- the three entry points ---------------------------------------------
    def _x_bf16(self, x, K: int, batch: bool):
        """x (bf16 host array) zero-padded to K columns, as a CUDA bf16 tensor."""
        xa = _host_array(x)
        bits = np.ascontiguousarray(xa).view(np.uint16)
        if batch:
            pad = np.zeros((bits.shape[0], K), dtype=np.uint16)
            pad[:, :bits.shape[1]] = bits
        else:
            pad = np.zeros(K, dtype=np.uint16)
            pad[:bits.shape[0]] = bits
        return torch.from_numpy(pad.view(np.int16)).to(torch.device("cuda", self.device)).view(torch.bfloat16)

    @staticmethod
    def _to_host_bf16(y) -> np.ndarray:
        return y.cpu().view(torch.int16).numpy().view(_bf16_type())

    def run_gemv_npu(self, W_combined, x_bf16) -> np.ndarray:
        """bf16 y (N,) = W x for a packed (N, K/32*20) matrix (model.py:283-361)."""
        w = self.resident(W_combined)
        from .ops import gemv_q_npu
        x = self._x_bf16(x_bf16, w.K, batch=False)
        y = torch.empty(w.N, dtype=torch.bfloat16, device=x.device)
        gemv_q_npu(w, x, y, N=w.N, K=w.K)
        return self._to_host_bf16(y)

    def run_ffn_fused_npu(self, l: int, x_bf16) -> np.ndarray:
        """bf16 y (H,) = FFN of layer l (model.py:363-397); the layer must be
        registered with register_ffn_layer."""
        w = self.layer_ffn.get(l)
        if w is None:
            raise KeyError(f"FFN layer {l} is not registered (register_ffn_layer)")
        from .ops import ffn_fused_npu
        x = self._x_bf16(x_bf16, w.H, batch=False)
        y = torch.empty((1, w.H), dtype=torch.bfloat16, device=x.device)
        ffn_fused_npu(w, x, y, H=w.H, I=w.I, activation=w.activation)
        return self._to_host_bf16(y[0])

    def run_gemm_npu(self, W_combined, x_bf16) -> np.ndarray:
        """bf16 Y (B, N) = X W^T for a packed matrix and bf16 X (B, <=K)
        (model.py:399-485)."""
        w = self.resident(W_combined)
        from .ops import gemm_q_npu
        x = self._x_bf16(x_bf16, w.K, batch=True)
        B = x.shape[0]
        y = torch.empty((B, w.N), dtype=torch.bfloat16, device=x.device)
        gemm_q_npu(w, x, y, B=B, N=w.N, K=w.K)
        return self._to_host_bf16(y)
