"""Model constants and launch-size limits (kernels/utils.py:11-46 of the reference)."""

from __future__ import annotations

import torch

# ZImage model dimensions (kernels/utils.py:11-14)
ZIMAGE_DIM = 3840
ZIMAGE_FFN_DIM = 10240
ZIMAGE_HEAD_DIM = 128
ZIMAGE_N_HEADS = 30

MAX_FUSED_SIZE = 65536  # kernels/utils.py:32


def check_row_size(n: int) -> None:
    """Raise RuntimeError for rows longer than the fused maximum (kernels/utils.py:33-37)."""
    if n > MAX_FUSED_SIZE:
        raise RuntimeError(
            f"Cannot launch kernel since n = {n} exceeds the maximum fused size = {MAX_FUSED_SIZE}.")


def require_bf16(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t.dtype != torch.bfloat16:
            raise ValueError(f"zimage_b200 kernels compute in bfloat16; got {t.dtype}")


def get_device_info() -> dict:
    """Device summary used in bench records (kernels/utils.py:61-84)."""
    if not torch.cuda.is_available():
        return {"available": False}
    dev = torch.cuda.current_device()
    props = torch.cuda.get_device_properties(dev)
    cap = torch.cuda.get_device_capability(dev)
    return {
        "available": True,
        "name": props.name,
        "compute_capability": f"{cap[0]}.{cap[1]}",
        "is_sm100": cap == (10, 0),
        "total_memory_gb": round(props.total_memory / (1024 ** 3), 2),
        "multi_processor_count": props.multi_processor_count,
        "cuda_version": torch.version.cuda or "unknown",
        "torch_version": torch.__version__,
    }
