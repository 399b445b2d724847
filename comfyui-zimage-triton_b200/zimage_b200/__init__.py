"""zimage_b200: sm_100a (B200) kernels for the Z-Image S3-DiT W8A8 forward path.

Drop-in for the hot path of the ComfyUI node "ZImage Triton Accelerate":
the same op names (``triton_rms_norm`` ...), the same INT8 quantisation
entry points and the same NextDiT patching function, backed by
``libzimage_b200.so`` (hand-written CUDA for sm_100a, C ABI in
``include/zimage_b200.h``).  There is no CPU or Triton path.
"""

__version__ = "0.1.0"

from .kernels import (  # noqa: E402
    TritonAdaLNModulation,
    TritonRMSNorm,
    TritonSwiGLU,
    triton_adaln_modulation,
    triton_fused_norm_gate_residual,
    triton_fused_qknorm_rope,
    triton_rms_norm,
    triton_rope_3d,
    triton_swiglu_forward,
)
from .patching import apply_triton_kernels_comfyui  # noqa: E402
from .quantization import apply_int8_quantization, restore_int8_quantization  # noqa: E402

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
    "apply_triton_kernels_comfyui",
    "apply_int8_quantization",
    "restore_int8_quantization",
]
