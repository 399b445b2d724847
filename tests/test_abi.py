"""The C ABI: library loads, exports exactly what include/*.h declares, validates on the host."""

import ctypes
import re

import pytest

from conftest import ROOT
from zimage_b200 import _lib


def _declared():
    out = {}
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        for m in re.finditer(r"ZIB_API\s+[\w\s\*]+?\b(zib_\w+)\s*\(([^)]*)\)", text, re.S):
            params = m.group(2).strip()
            n = 0 if params in ("", "void") else len(params.split(","))
            out[m.group(1)] = n
    return out


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    decl = _declared()
    assert len(decl) >= 19
    for name, nparams in decl.items():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, name
        assert len(_lib.SIGNATURES[name]) == nparams, name
    assert set(_lib.SIGNATURES) == set(decl)


def test_version_and_status_strings():
    lib = _lib.load()
    assert lib.zib_version() == 100
    assert lib.zib_status_string(0) == b"ok"
    assert lib.zib_status_string(6).startswith(b"bounded")


def test_host_validation_before_launch():
    lib = _lib.load()
    # null operands are rejected on the host, no device needed
    assert lib.zib_act_quant(None, 128, None, 128, None, None, 4, 128, 1, None) == _lib.ZIB_ERR_INVALID_ARG
    # K not a multiple of 128 with the Hadamard rotation
    assert lib.zib_act_quant(16, 200, 16, 200, 16, None, 4, 200, 1, None) == _lib.ZIB_ERR_INVALID_ARG
    # misaligned GEMM K
    assert lib.zib_gemm_w8a8(16, 24, 16, 24, 16, 16, None, 16, 8, 4, 8, 24, None) == _lib.ZIB_ERR_ALIGNMENT
    assert lib.zib_qknorm_rope(16, 0, 0, 0, 16, 0, 0, 0, 16, 16, 0, None, 1, 1, 1, 64, 1e-5, None) == \
        _lib.ZIB_ERR_INVALID_ARG
    # fused-epilogue GEMMs: features not a multiple of the 128-group; odd head count
    assert lib.zib_gemm_w8a8_swiglu_had(16, 128, 16, 16, 128, 16, 16, 16, 16, 200, 8, 200, 128, None) == \
        _lib.ZIB_ERR_INVALID_ARG
    assert lib.zib_gemm_w8a8_qk_norm_rope(16, 128, 16, 128, 16, 16, 16, 1152, 8, 1152, 128, 16, 16, 1e-5, 1e-5,
                                          16, 16, 0, 8, 3, None) == _lib.ZIB_ERR_INVALID_ARG
    # M not a multiple of the sequence length
    assert lib.zib_gemm_w8a8_qk_norm_rope(16, 128, 16, 128, 16, 16, 16, 768, 9, 768, 128, 16, 16, 1e-5, 1e-5,
                                          16, 16, 0, 8, 2, None) == _lib.ZIB_ERR_INVALID_ARG
    # the one-tensor [w1; w3] SwiGLU GEMM: ragged features, null weight
    assert lib.zib_gemm_w8a8_swiglu_had_w13(16, 128, 16, 128, 16, 16, 16, 16, 200, 8, 200, 128, None) == \
        _lib.ZIB_ERR_INVALID_ARG
    assert lib.zib_gemm_w8a8_swiglu_had_w13(16, 128, None, 128, 16, 16, 16, 16, 128, 8, 128, 128, None) == \
        _lib.ZIB_ERR_INVALID_ARG
    # misaligned output of the SwiGLU epilogue
    assert lib.zib_gemm_w8a8_swiglu_had(16, 128, 16, 16, 128, 16, 16, 16, 18, 128, 8, 128, 128, None) == \
        _lib.ZIB_ERR_ALIGNMENT
    # split-K workspace registration: both buffers or neither, at least one partial-tile pair, aligned
    pair = 2 * 128 * 256 * 4
    assert lib.zib_gemm_set_split_workspace(0, 4096, pair, None, 2) == _lib.ZIB_ERR_INVALID_ARG
    assert lib.zib_gemm_set_split_workspace(0, 4096, pair - 16, 8192, 2) == _lib.ZIB_ERR_INVALID_ARG
    assert lib.zib_gemm_set_split_workspace(0, 4100, pair, 8192, 2) == _lib.ZIB_ERR_ALIGNMENT
    assert lib.zib_gemm_set_split_workspace(64, 4096, pair, 8192, 2) == _lib.ZIB_ERR_INVALID_ARG
    assert lib.zib_gemm_set_split_workspace(0, None, 0, None, 0) == _lib.ZIB_OK  # nothing registered
    with pytest.raises(ValueError):
        _lib.check(_lib.ZIB_ERR_INVALID_ARG, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ZIB_ERR_TIMEOUT, "x")


def test_ops_refuse_cpu_tensors():
    import torch
    from zimage_b200 import triton_rms_norm, triton_swiglu_forward

    x = torch.zeros(2, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        triton_rms_norm(x, torch.ones(8))
    with pytest.raises(ValueError, match="same shape"):
        triton_swiglu_forward(x, torch.zeros(2, 4, dtype=torch.bfloat16))
