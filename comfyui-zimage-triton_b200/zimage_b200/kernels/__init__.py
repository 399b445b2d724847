"""sm_100a kernels behind the reference's op-level names (kernels/__init__.py:3-27)."""

from .adaln_modulation import TritonAdaLNModulation, triton_adaln_modulation
from .fused_norm_residual import triton_fused_norm_gate_residual
from .fused_qknorm_rope import triton_fused_qknorm_rope
from .rms_norm import TritonRMSNorm, triton_rms_norm
from .rope_3d import triton_rope_3d
from .swiglu import TritonSwiGLU, triton_swiglu_forward

__all__ = [
    "triton_rms_norm",
    "TritonRMSNorm",
    "triton_swiglu_forward",
    "TritonSwiGLU",
    "triton_rope_3d",
    "triton_adaln_modulation",
    "TritonAdaLNModulation",
    "triton_fused_norm_gate_residual",
    "triton_fused_qknorm_rope",
]
