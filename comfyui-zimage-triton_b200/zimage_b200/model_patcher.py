"""ComfyUI ModelPatcher glue for INT8 models (model_patcher.py of the reference).

Only importable inside ComfyUI (needs ``comfy``).  Keeps INT8 module weights
on CPU during LoRA patching and skips INT8 modules in partial offload, keyed
on the same ``_int8_quantized`` flag (model_patcher.py:31-110).
"""

from __future__ import annotations

import comfy.utils  # noqa: F401  (ImportError outside ComfyUI is expected)
from comfy.model_patcher import ModelPatcher


class ZImageTritonModelPatcher(ModelPatcher):
    def _is_int8_key(self, key: str) -> bool:
        parts = key.rsplit(".", 1)
        if len(parts) < 2:
            return False
        try:
            module = comfy.utils.get_attr(self.model, parts[0])
            return getattr(module, "_int8_quantized", False)
        except (AttributeError, KeyError):
            return False

    def patch_weight_to_device(self, key, device_to=None, inplace_update=False, return_weight=False):
        if self._is_int8_key(key):
            device_to = None
        return super().patch_weight_to_device(key, device_to=device_to, inplace_update=inplace_update,
                                              return_weight=return_weight)

    def _refresh_int8(self) -> None:
        dm = getattr(getattr(self.model, "diffusion_model", None), "_int8_lora_aware", False)
        if dm:
            from zimage_b200.quantization import refresh_int8_weights

            refresh_int8_weights(self.model.diffusion_model)

    def patch_model(self, *args, **kwargs):
        # LoRA-aware INT8: the patches just written into the (CPU) source weights are
        # re-quantised into the layers' int8 buffers
        out = super().patch_model(*args, **kwargs)
        self._refresh_int8()
        return out

    def unpatch_model(self, *args, **kwargs):
        out = super().unpatch_model(*args, **kwargs)
        self._refresh_int8()
        return out

    def partially_unload(self, device_to, memory_to_free=0, force_patch_weights=False):
        saved = []
        for _n, m in self.model.named_modules():
            if getattr(m, "_int8_quantized", False) and getattr(m, "comfy_patched_weights", False):
                m.comfy_patched_weights = False
                saved.append(m)
        try:
            return super().partially_unload(device_to, memory_to_free, force_patch_weights)
        finally:
            for m in saved:
                m.comfy_patched_weights = True


def upgrade_model_patcher(model) -> None:  # noqa: ANN001
    if not isinstance(model, ZImageTritonModelPatcher):
        model.__class__ = ZImageTritonModelPatcher
