"""INT8 W8A8 (+ Hadamard) quantisation (quantization/__init__.py of the reference)."""

from .int8_linear import apply_int8_quantization, refresh_int8_weights, restore_int8_quantization

__all__ = ["apply_int8_quantization", "restore_int8_quantization", "refresh_int8_weights"]
