"""alveare_b200: B200-native (sm_100a) Q4 decode hot path of Alveare.

Hand-written CUDA kernels behind a C ABI (include/alveare_b200.h) with the
reference's operator signatures on top (``alveare_b200.ops``).
"""
from .ops import (FusedFFNWeight, Q4Weight, ffn_fused_npu, gemm_q_npu, gemv_q_npu,
                  pack_ffn_fused_weights, q4_quantize)

__all__ = ["Q4Weight", "FusedFFNWeight", "gemv_q_npu", "ffn_fused_npu", "gemm_q_npu",
           "pack_ffn_fused_weights", "q4_quantize"]
