"""ComfyUI node "ZImage Triton Accelerate" backed by the sm_100a kernels.

Same node contract as the reference (nodes.py:92-242): class
``ZImageTritonApply``, inputs ``model: MODEL`` and optional
``enable_int8: BOOLEAN`` (default True), returns the same model object
mutated in place, idempotent per config tuple, restore-before-repatch.
"""

from __future__ import annotations

import logging

logger = logging.getLogger(__name__)


def _restore_original_forwards(transformer) -> None:  # noqa: ANN001
    """Undo every patch (nodes.py:10-56): INT8 modules, forwards, SwiGLU gating, RMSNorm modules."""
    import torch.nn as nn

    if getattr(transformer, "_int8_quantized", False):
        from zimage_b200.quantization import restore_int8_quantization

        n = restore_int8_quantization(transformer)
        logger.info("[ZImage-B200] Restored %d INT8-quantized modules.", n)

    for module in transformer.modules():
        if hasattr(module, "_original_forward"):
            module.forward = module._original_forward
            delattr(module, "_original_forward")
        if hasattr(module, "_original_silu_gating"):
            module._forward_silu_gating = module._original_silu_gating
            delattr(module, "_original_silu_gating")
        for key in ("_zib_cache", "_zib_next", "_zib_fused_ok", "_zib_adaln_stack"):
            module.__dict__.pop(key, None)

    for name, child in list(transformer.named_modules()):
        original = getattr(child, "_original_module", None)
        if original is not None:
            parts = name.split(".")
            parent: nn.Module = transformer
            for part in parts[:-1]:
                parent = getattr(parent, part)
            setattr(parent, parts[-1], original)

    transformer._triton_patched = False
    transformer._triton_config = None
    logger.info("[ZImage-B200] Restored original forwards.")


def _log_patch_state(transformer, label: str) -> None:  # noqa: ANN001
    """Debug counts of patched modules (nodes.py:59-89)."""
    n_fwd = n_silu = n_norm = n_layers = 0
    for m in transformer.modules():
        n_fwd += hasattr(m, "_original_forward")
        n_silu += hasattr(m, "_original_silu_gating")
        n_norm += type(m).__name__ == "TritonRMSNorm"
        n_layers += type(m).__name__ == "JointTransformerBlock"
    logger.debug("[ZImage-B200] %s: layers=%d, _triton_patched=%s, config=%s, _original_forward=%d, "
                 "_original_silu=%d, TritonRMSNorm=%d", label, n_layers,
                 getattr(transformer, "_triton_patched", False), getattr(transformer, "_triton_config", None),
                 n_fwd, n_silu, n_norm)


class ZImageTritonApply:
    """Apply the sm_100a kernels (+ W8A8 + Hadamard INT8) to a Z-Image S3-DiT model."""

    @classmethod
    def INPUT_TYPES(cls):
        return {
            "required": {
                "model": ("MODEL",),
            },
            "optional": {
                "enable_int8": (
                    "BOOLEAN",
                    {
                        "default": True,
                        "tooltip": "Enable W8A8+Hadamard INT8 quantization (tcgen05 int8 GEMM). "
                                   "OFF: bf16 linears with the fused elementwise kernels only.",
                    },
                ),
            },
        }

    RETURN_TYPES = ("MODEL",)
    RETURN_NAMES = ("model",)
    FUNCTION = "apply_triton"
    CATEGORY = "ZImage-Triton"
    DESCRIPTION = ("Accelerate ZImage S3-DiT on B200 (sm_100a) with hand-written CUDA kernels + "
                   "W8A8/Hadamard INT8 on tcgen05 tensor cores.")

    # Internal kernel defaults, not exposed to the UI (nodes.py:151-156)
    enable_fused_norm = True
    enable_swiglu = True
    enable_fused_qknorm_rope = True
    enable_fused_adaln = False
    enable_fused_norm_residual = True
    # INT8 policy knobs beyond the reference node (defaults = reference policy)
    int8_min_dim = 1024
    int8_skip_sensitive = True
    int8_policy = None  # "reference" / "all_linears" / "main_layers"; None: from int8_skip_sensitive
    # re-quantise INT8 layers whose bf16 weight a LoRA patch changed (the reference ignores LoRA there)
    int8_lora_aware = False

    def apply_triton(self, model, enable_int8: bool = True):  # noqa: ANN001
        from zimage_b200.patching import apply_triton_kernels_comfyui

        transformer = model.model.diffusion_model
        if not hasattr(transformer, "layers"):
            logger.warning("[ZImage-B200] Model does not appear to be ZImage/Lumina2 (no .layers "
                           "attribute). Skipping patching.")
            return (model,)

        _log_patch_state(transformer, "pre-patch")
        current_config = (
            self.enable_fused_norm,
            self.enable_swiglu,
            self.enable_fused_qknorm_rope,
            self.enable_fused_adaln,
            self.enable_fused_norm_residual,
            enable_int8,
        )
        prev_config = getattr(transformer, "_triton_config", None)
        if getattr(transformer, "_triton_patched", False):
            if prev_config == current_config:
                logger.info("[ZImage-B200] Already patched with same config, skipping.")
                return (model,)
            logger.info("[ZImage-B200] Config changed (%s -> %s), restoring originals before re-patching.",
                        prev_config, current_config)
            _restore_original_forwards(transformer)

        stats = apply_triton_kernels_comfyui(
            transformer,
            enable_fused_norm=self.enable_fused_norm,
            enable_swiglu=self.enable_swiglu,
            enable_fused_qknorm_rope=self.enable_fused_qknorm_rope,
            enable_fused_adaln=self.enable_fused_adaln,
            enable_fused_norm_residual=self.enable_fused_norm_residual,
        )
        transformer._triton_patched = True
        transformer._triton_config = current_config
        transformer._triton_stats = stats
        _log_patch_state(transformer, "post-patch")
        logger.info("[ZImage-B200] Applied kernels: %s", stats)

        if enable_int8 and not getattr(transformer, "_int8_quantized", False):
            from zimage_b200.quantization import apply_int8_quantization

            int8_stats = apply_int8_quantization(transformer, min_dim=self.int8_min_dim, mode="w8a8_hadamard",
                                                 skip_sensitive=self.int8_skip_sensitive, policy=self.int8_policy,
                                                 lora_aware=self.int8_lora_aware)
            transformer._int8_quantized = True
            transformer._int8_stats = int8_stats
            # ComfyUI VRAM accounting: recompute the model size (nodes.py:217-223)
            model.size = 0
            try:  # ComfyUI-only ModelPatcher upgrade (model_patcher.py of the reference)
                from zimage_b200.model_patcher import upgrade_model_patcher

                upgrade_model_patcher(model)
            except ImportError:
                pass
            logger.info("[ZImage-B200] INT8 W8A8+Hadamard: %s", int8_stats)
        return (model,)
