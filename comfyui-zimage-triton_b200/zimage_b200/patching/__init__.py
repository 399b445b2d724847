"""Module-replacement surface for ComfyUI's NextDiT (models/patching_comfyui.py of the reference)."""

from .patching_comfyui import apply_triton_kernels_comfyui, fused_block_forward

__all__ = ["apply_triton_kernels_comfyui", "fused_block_forward"]
