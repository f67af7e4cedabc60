"""m5kernels_b200 — B200-native (sm_100a) quantized linear-projection hot path.

The `cuda-b200` backend of the m5kernels operator contracts:
    quantize, gemm                     (twin of m5kernels.metal)
    gemm_schedule                      (the schedule `m5bench tune` sweeps, in place of Metal tiles)
    rotate, hadamard_quantize          (twin of m5kernels.hadamard)
    fused_norm_hadamard_quantize,
    fused_gated_residual_norm_hadamard_quantize,
    gated_residual_add, unfused_norm   (twin of m5kernels.norm_hadamard)
    projection_qk_rope, qk_norm_rope   (twin of m5kernels.qk_rope)
    projection_qkv_rope                (grouped Q/K/V layout of the H3 integration)
    rms_quantize                       (twin of m5kernels.rms_quant)
    linear, OnlineProjection           (the online quantize -> gemm stage in one call / bound step)
All of them run hand-written CUDA kernels from libm5b200.so through its C ABI
(include/m5b200.h); there is no CPU fallback.
"""

from .cuda import gemm, gemm_allgather, gemm_schedule, quantize
from .hadamard import SUPPORTED_BLOCK_SIZES, hadamard_quantize, rotate
from .linear import OnlineProjection, linear
from .norm_hadamard import (fused_gated_residual_norm_hadamard_quantize,
                            fused_norm_hadamard_quantize, gated_residual_add, unfused_norm)
from .qk_rope import (grouped_qkv_weights, projection_qk_rope, projection_qkv_rope, qk_norm_rope,
                      rope_tables)
from .rms_quant import rms_quantize

__all__ = [
    "gemm", "gemm_allgather", "gemm_schedule", "quantize", "rotate", "hadamard_quantize", "SUPPORTED_BLOCK_SIZES",
    "fused_norm_hadamard_quantize", "fused_gated_residual_norm_hadamard_quantize",
    "projection_qk_rope", "rope_tables", "linear", "rms_quantize", "gated_residual_add",
    "unfused_norm", "qk_norm_rope", "projection_qkv_rope", "grouped_qkv_weights",
    "OnlineProjection",
]
