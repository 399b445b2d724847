"""ctypes binding of libzimage_b200.so (the sm_100a kernels behind every op).

There is no CPU or eager fallback: if the library is missing, or a tensor is
not on an sm_100 CUDA device, the call raises.  Status codes of the C ABI are
mapped to the exceptions the reference raises for the same conditions
(ValueError for shape/dtype problems, ``kernels/swiglu.py:82-86``;
RuntimeError for oversize rows, ``kernels/utils.py:33-37``).
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libzimage_b200.so")

ZIB_OK = 0
ZIB_ERR_INVALID_ARG = 1
ZIB_ERR_ALIGNMENT = 2
ZIB_ERR_UNSUPPORTED = 3
ZIB_ERR_LAUNCH = 4
ZIB_ERR_TOO_LARGE = 5
ZIB_ERR_TIMEOUT = 6

_VP, _I64, _I32, _F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
_FP = ctypes.POINTER(ctypes.c_float)

# name -> argtypes (all return int status unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "zib_version": [],
    "zib_status_string": [_I32],
    "zib_last_error": [],
    "zib_device_check": [_I32],
    "zib_device_error_read_clear": [],
    "zib_selftest_bounded_wait": [_VP],
    "zib_act_quant": [_VP, _I64, _VP, _I64, _VP, _VP, _I64, _I64, _I32, _VP],
    "zib_gemm_w8a8": [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I64, _VP],
    "zib_gemm_w8a8_acc_i32": [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _I64, _VP],
    "zib_gemm_w8a8_swiglu_had": [_VP, _I64, _VP, _VP, _I64, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I64, _VP],
    "zib_gemm_w8a8_swiglu_had_w13": [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I64, _VP],
    "zib_gemm_w8a8_qk_norm_rope": [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _I64, _I64, _I64, _I64, _VP, _VP,
                                   _F32, _F32, _VP, _VP, _I64, _I64, _I64, _VP],
    "zib_gemm_set_variant": [_I32],
    "zib_gemm_set_split": [_I32],
    "zib_gemm_set_group_budget": [_I64],
    "zib_gemm_set_split_workspace": [_I32, _VP, _I64, _VP, _I64],
    "zib_gemm_w8a8_static_scratch": [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _VP, _I64, _I64, _I64, _I64, _I32, _VP],
    "zib_weight_prep": [_VP, _I64, _VP, _I64, _VP, _VP, _VP, _I64, _I64, _I64, _I32, _VP],
    "zib_rms_norm": [_VP, _I64, _VP, _VP, _I64, _I64, _I64, _F32, _VP],
    "zib_rmsnorm_mod": [_VP, _I64, _VP, _VP, _VP, _I64, _I64, _VP, _I64, _I64, _I64, _F32, _VP],
    "zib_rmsnorm_mod_quant": [_VP, _I64, _VP, _VP, _VP, _I64, _I64, _VP, _I64, _VP, _I64, _I64, _F32,
                              _I32, _VP],
    "zib_norm_gate_residual": [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _VP, _VP, _I64, _I64, _I64, _F32,
                               _VP],
    "zib_norm_gate_residual_mod_quant": [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _VP, _VP, _I64, _VP, _VP,
                                         _VP, _I64, _VP, _I64, _VP, _I64, _I64, _F32, _F32, _I32, _VP],
    "zib_norm_gate_residual_mod_quant_w16": [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _VP, _VP, _I64, _VP,
                                             _VP, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _F32, _F32, _I32,
                                             _VP],
    "zib_swiglu": [_VP, _I64, _VP, _I64, _VP, _I64, _I64, _I64, _VP],
    "zib_swiglu_quant": [_VP, _I64, _VP, _I64, _VP, _I64, _VP, _I64, _I64, _I32, _VP],
    "zib_qknorm_rope": [_VP, _I64, _I64, _I64, _VP, _I64, _I64, _I64, _VP, _VP, _I64, _VP, _I64, _I64,
                        _I64, _I64, _F32, _VP],
    "zib_adaln_modulation": [_VP, _I64, _VP, _VP, _VP, _VP, _I64, _I64, _VP],
    "zib_adaln_gates": [_VP, _I64, _VP, _I64, _I64, _VP],
}
_RESTYPES = {"zib_status_string": ctypes.c_char_p, "zib_last_error": ctypes.c_char_p}

_lib = None
_lock = threading.Lock()
_checked_devices: set[int] = set()


def load() -> ctypes.CDLL:
    """Load the library once and declare every exported symbol."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run "
                    "`python comfyui-zimage-triton_b200/csrc/build.py` (nvcc, sm_100a)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, argtypes in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = argtypes
                fn.restype = _RESTYPES.get(name, ctypes.c_int)
            _lib = lib
    return _lib


def last_error() -> str:
    return load().zib_last_error().decode(errors="replace")


def check(status: int, what: str) -> None:
    if status == ZIB_OK:
        return
    lib = load()
    msg = f"{what}: {lib.zib_status_string(status).decode()}: {last_error()}"
    if status in (ZIB_ERR_INVALID_ARG, ZIB_ERR_ALIGNMENT):
        raise ValueError(msg)
    raise RuntimeError(msg)


def require_device(t: torch.Tensor) -> int:
    """Raise unless ``t`` lives on an sm_100 CUDA device; returns the device index."""
    if not t.is_cuda:
        raise ValueError(
            "zimage_b200 ops run only on CUDA tensors (sm_100a); got a tensor on "
            f"{t.device}. There is no CPU path.")
    dev = t.device.index if t.device.index is not None else torch.cuda.current_device()
    if dev not in _checked_devices:
        check(load().zib_device_check(dev), "device check")
        _checked_devices.add(dev)
    return dev


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


# Number of kernel-launching entry points called through ``call`` (the
# benchmark reports it as its launch count).
LAUNCHES = 0


# Split-K workspaces of the plain GEMM entry points, one per device: allocated here with torch
# (so the memory is the framework's, and the library itself never allocates) and registered
# with zib_gemm_set_split_workspace on a device's first such GEMM.  256 KB of partial tiles per
# CTA pair (one per two SMs) plus two zeroed arrival counters per tail tile.
_SPLIT_WS: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
_SPLIT_GEMMS = ("zib_gemm_w8a8", "zib_gemm_w8a8_acc_i32")


def ensure_split_workspace(dev: int | None = None) -> None:
    dev = torch.cuda.current_device() if dev is None else dev
    if dev in _SPLIT_WS:
        return
    pairs = max(1, torch.cuda.get_device_properties(dev).multi_processor_count // 2)
    ws = torch.empty(pairs * 2 * 128 * 256, dtype=torch.int32, device=f"cuda:{dev}")
    ctr = torch.zeros(pairs * 2, dtype=torch.int32, device=f"cuda:{dev}")
    check(load().zib_gemm_set_split_workspace(dev, ws.data_ptr(), ws.numel() * 4, ctr.data_ptr(), ctr.numel()),
          "zib_gemm_set_split_workspace")
    _SPLIT_WS[dev] = (ws, ctr)


def call(name: str, *args) -> None:
    """Invoke ``name`` and raise on a non-zero status."""
    global LAUNCHES
    if name in _SPLIT_GEMMS:
        ensure_split_workspace()
    LAUNCHES += 1
    check(getattr(load(), name)(*args), name)


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def device_error_read_clear() -> int:
    """Synchronising read of the device error word (ZIB_ERR_TIMEOUT after an expired wait)."""
    return int(load().zib_device_error_read_clear())


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
