"""Host logic that needs no GPU: INT8 layer selection, patch surface, node contract."""

import json

import torch

from conftest import GOLDEN
from helpers import ztree


def test_int8_layer_selection_matches_reference():
    from zimage_b200.quantization.int8_linear import select_layers

    gold = json.loads((GOLDEN / "policy.json").read_text())
    plan, stats = select_layers(ztree(), min_dim=0, mode="w8a8_hadamard")
    assert stats == gold["stats"]
    assert sorted(n for n, _m, _h in plan) == gold["quantized"]
    assert all(h for _n, _m, h in plan)


def test_int8_selection_min_dim_and_policy_knobs():
    from zimage_b200.quantization.int8_linear import select_layers

    _plan, st = select_layers(ztree(), min_dim=1024, mode="w8a8_hadamard")
    assert st["quantized"] == 0 and st["skipped"] > 0
    plan, st = select_layers(ztree(), min_dim=0, mode="w8a8_hadamard", skip_sensitive=False)
    assert st["sensitive"] == 0 and st["quantized"] == len(plan)
    assert any(not h for _n, _m, h in plan)  # x_embedder (in=64) has no Hadamard
    assert st["had_skipped"] >= 1


def test_patch_stats_match_reference():
    from zimage_b200 import apply_triton_kernels_comfyui

    gold = json.loads((GOLDEN / "patch_stats.json").read_text())
    assert apply_triton_kernels_comfyui(ztree(), enable_fused_adaln=False) == gold


class _FakeModelPatcher:
    def __init__(self, dm):
        class _M:
            pass

        self.model = _M()
        self.model.diffusion_model = dm
        self.size = 123


def test_node_contract_and_idempotent_patch_restore():
    import nodes
    from zimage_b200.kernels.rms_norm import TritonRMSNorm

    spec = nodes.ZImageTritonApply.INPUT_TYPES()
    assert spec["required"] == {"model": ("MODEL",)}
    assert spec["optional"]["enable_int8"][0] == "BOOLEAN"
    assert spec["optional"]["enable_int8"][1]["default"] is True
    assert nodes.ZImageTritonApply.RETURN_TYPES == ("MODEL",)
    assert nodes.ZImageTritonApply.FUNCTION == "apply_triton"
    assert nodes.ZImageTritonApply.CATEGORY == "ZImage-Triton"

    tree = ztree()
    mp = _FakeModelPatcher(tree)
    node = nodes.ZImageTritonApply()
    (out,) = node.apply_triton(mp, enable_int8=False)
    assert out is mp
    assert tree._triton_patched and tree._triton_config == (True, True, True, False, True, False)
    n_norm = sum(isinstance(m, TritonRMSNorm) for m in tree.modules())
    assert n_norm == 60
    blk = tree.layers[1]
    assert "forward" in blk.__dict__ and hasattr(blk, "_original_forward")
    # same config -> no-op
    node.apply_triton(mp, enable_int8=False)
    assert sum(isinstance(m, TritonRMSNorm) for m in tree.modules()) == n_norm
    # restore brings the original modules back
    nodes._restore_original_forwards(tree)
    assert not any(isinstance(m, TritonRMSNorm) for m in tree.modules())
    # like the reference, restore re-binds the saved original bound method
    assert blk.forward.__func__ is type(blk).forward and not hasattr(blk, "_original_forward")
    assert not hasattr(tree.layers[1].feed_forward, "_original_silu_gating")


def test_node_skips_non_zimage_models():
    import nodes

    mp = _FakeModelPatcher(torch.nn.Linear(2, 2))
    (out,) = nodes.ZImageTritonApply().apply_triton(mp)
    assert out is mp


def test_registration_names():
    import importlib.util
    import sys

    from conftest import ROOT

    spec = importlib.util.spec_from_file_location(
        "zimage_node_pkg", ROOT / "comfyui-zimage-triton_b200" / "__init__.py",
        submodule_search_locations=[str(ROOT / "comfyui-zimage-triton_b200")])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["zimage_node_pkg"] = mod
    spec.loader.exec_module(mod)
    assert list(mod.NODE_CLASS_MAPPINGS) == ["ZImageTritonApply"]
    assert mod.NODE_DISPLAY_NAME_MAPPINGS == {"ZImageTritonApply": "ZImage Triton Accelerate"}


def test_ffn_weights_become_halves_of_one_tensor():
    """The fused block path puts w1 and w3 into one [2F, K] tensor once and makes the modules'
    buffers views of its halves (no second copy); it finds the halves again afterwards, and
    keeps the two-weight GEMM when the weights cannot share a tensor (checked on the host)."""
    import types

    from zimage_b200.patching.patching_comfyui import _w13_halves

    def ffn(w1, w3):
        ff = types.SimpleNamespace(w1=torch.nn.Module(), w3=torch.nn.Module())
        ff.w1.register_buffer("_w_int8", w1)
        ff.w3.register_buffer("_w_int8", w3)
        return ff

    g = torch.Generator().manual_seed(0)
    w1 = torch.randint(-127, 128, (64, 128), generator=g, dtype=torch.int8)
    w3 = torch.randint(-127, 128, (64, 128), generator=g, dtype=torch.int8)
    ff = ffn(w1.clone(), w3.clone())
    w13 = _w13_halves(ff)
    assert w13.shape == (128, 128) and torch.equal(w13, torch.cat([w1, w3]))
    assert ff.w1._w_int8.data_ptr() == w13.data_ptr() and torch.equal(ff.w1._w_int8, w1)
    assert ff.w3._w_int8.data_ptr() == w13.data_ptr() + 64 * 128 and torch.equal(ff.w3._w_int8, w3)
    assert _w13_halves(ff) is w13                                            # found again, no new copy
    assert _w13_halves(ffn(w1[:, :120], w3[:, :120])) is None                # K not a multiple of 16
    assert _w13_halves(ffn(w1[:, ::2], w3[:, ::2])) is None                  # column-strided
    assert _w13_halves(ffn(w1[:32], w3)) is None                             # different shapes


def test_weight_fingerprint_sees_in_place_updates():
    """The LoRA-aware refresh keys on (pointer, version, sampled values): an in-place
    low-rank update through .data (no version bump) and a write to the last element both
    change it; the sampled positions stay in range for any size."""
    from zimage_b200.quantization.int8_linear import weight_fingerprint

    for shape in [(11520, 3840), (3, 5), (4096, 1), (1, 1)]:
        w = torch.zeros(shape, dtype=torch.bfloat16)
        fp = weight_fingerprint(w)
        w.data[-1, -1] = 1.0
        assert weight_fingerprint(w) != fp and w._version == 0
    w = torch.randn(1024, 512).to(torch.bfloat16)
    fp = weight_fingerprint(w)
    assert weight_fingerprint(w) == fp
    g = torch.Generator().manual_seed(0)
    w.data.copy_((w.float() + 0.05 * torch.randn(1024, 4, generator=g) @ torch.randn(4, 512, generator=g))
                 .to(torch.bfloat16))
    assert weight_fingerprint(w) != fp
