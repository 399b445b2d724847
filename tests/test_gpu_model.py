"""Module-level parity on the GPU: W8A8 linear module, patched block, multi-layer step."""

import pytest
import torch

from conftest import GOLDEN
from helpers import max_abs, rel_l2
from oracle import model as omodel
from oracle import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["bias", "nobias"])
def test_w8a8_module_vs_reference_fixture(cuda, case):
    from zimage_b200 import apply_int8_quantization, restore_int8_quantization

    d = torch.load(GOLDEN / "w8a8_hadamard.pt")[case]
    N, K = d["w"].shape
    holder = torch.nn.Module()
    holder.proj = torch.nn.Linear(K, N, bias=d["b"] is not None, dtype=torch.bfloat16, device="cuda")
    with torch.no_grad():
        holder.proj.weight.copy_(d["w"])
        if d["b"] is not None:
            holder.proj.bias.copy_(d["b"])
    stats = apply_int8_quantization(holder, min_dim=0, mode="w8a8_hadamard")
    assert stats == d["stats"]
    lin = holder.proj
    assert lin._int8_quantized and lin._int8_use_hadamard and lin.weight.device.type == "cpu"
    owq, osw, _ = ops.weight_prep(d["w"])
    assert torch.equal(lin._w_int8.cpu(), owq) and torch.equal(lin._w_scale.cpu(), osw)
    assert int((lin._w_int8.cpu() != d["w_int8"]).sum()) <= 2
    y = lin(d["x"].cuda()).cpu()
    assert torch.equal(y, ops.w8a8_linear(d["x"], owq, osw, d["b"]))
    assert rel_l2(y, d["y"]) <= 5e-3
    assert (y != d["y"]).float().mean().item() <= 2e-3
    assert "proj.weight" not in holder.state_dict()
    assert restore_int8_quantization(holder) == 1
    assert not hasattr(lin, "_w_int8") and lin.weight.device.type == "cuda"


def test_w8a8_plain_module_vs_reference_fixture(cuda):
    from zimage_b200 import apply_int8_quantization

    d = torch.load(GOLDEN / "w8a8_plain.pt")["plain"]
    N, K = d["w"].shape
    holder = torch.nn.Module()
    holder.proj = torch.nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device="cuda")
    with torch.no_grad():
        holder.proj.weight.copy_(d["w"])
    apply_int8_quantization(holder, min_dim=0, mode="w8a8_hadamard")
    assert not holder.proj._int8_use_hadamard
    assert torch.equal(holder.proj._w_int8.cpu(), d["w_int8"])
    y = holder.proj(d["x"].cuda()).cpu()
    assert torch.equal(y, d["y"])


def _small_model(n_layers, dim, heads, ffn, seed=0):
    from zimage_b200.nextdit import NextDiT, load_layer_params

    gen = torch.Generator().manual_seed(seed)
    params = [omodel.make_layer_params(gen, dim=dim, ffn=ffn, n_heads=heads) for _ in range(n_layers)]
    m = NextDiT(n_layers=n_layers, dim=dim, n_heads=heads, ffn_dim=ffn, device="cuda")
    for blk, p in zip(m.layers, params):
        load_layer_params(blk, p)
    return m, params


def _inputs(B, gh, gw, n_txt, dim, seed=5):
    g = torch.Generator().manual_seed(seed)
    S = gh * gw + n_txt
    x = torch.randn(B, S, dim, generator=g).to(torch.bfloat16)
    t = torch.randn(B, 256, generator=g).to(torch.bfloat16)
    pos = ops.zimage_positions(gh, gw, n_txt)
    fm = ops.rope_freqs_matrix(pos).unsqueeze(0)          # [1, S, 64, 2, 2] (ComfyUI form)
    fc = ops.rope_freqs_complex(pos).unsqueeze(0)
    return x, t, fm, fc


class _MP:
    def __init__(self, dm):
        class _M:
            pass

        self.model = _M()
        self.model.diffusion_model = dm


def _patch(m, all_linears=True):
    import nodes

    node = nodes.ZImageTritonApply()
    if all_linears:
        node.int8_min_dim = 0
        node.int8_skip_sensitive = False
    node.apply_triton(_MP(m), enable_int8=True)
    return node


def test_block_fused_equals_composed_and_matches_oracle(cuda):
    from zimage_b200.patching import patching_comfyui as pc

    dim, heads, ffn = 1024, 8, 2816
    m, params = _small_model(1, dim, heads, ffn)
    _patch(m)
    x, t, fm, fc = _inputs(2, 8, 8, 16, dim)
    with torch.no_grad():
        y_fused = m(x.cuda(), t.cuda(), fm.cuda())
        pc.ENABLE_FUSED_BLOCK = False
        try:
            y_comp = m(x.cuda(), t.cuda(), fm.cuda())
        finally:
            pc.ENABLE_FUSED_BLOCK = True
    assert "_zib_cache" in m.layers[0].__dict__
    assert torch.equal(y_fused, y_comp)
    p = omodel.prep_layer(params[0], quant_adaln=True)
    want = omodel.block_forward(p, x, fc, t, n_heads=heads)
    y = y_fused.cpu()
    assert rel_l2(y, want) <= 5e-3
    assert max_abs(y, want) <= 2e-2 * max(1.0, want.abs().max().item())


def test_step_matches_oracle(cuda):
    dim, heads, ffn, L = 1024, 8, 2816, 3
    m, params = _small_model(L, dim, heads, ffn, seed=1)
    _patch(m)
    x, t, fm, fc = _inputs(2, 8, 8, 16, dim, seed=6)
    with torch.no_grad():
        y = m(x.cuda(), t.cuda(), fm.cuda()).cpu()
    want = omodel.step_forward([omodel.prep_layer(p, quant_adaln=True) for p in params], x, fc, t,
                               n_heads=heads)
    assert rel_l2(y, want) <= 5e-3
    assert max_abs(y, want) <= 2e-2 * max(1.0, want.abs().max().item())


def test_reference_policy_mixed_bf16_and_int8_layers(cuda):
    """Default node policy: layers.0 and adaLN stay bf16 (composed path), the rest fused."""
    dim, heads, ffn, L = 1024, 8, 2816, 4
    m, params = _small_model(L, dim, heads, ffn, seed=2)
    _patch(m, all_linears=False)
    st = m._int8_stats
    assert st["sensitive"] > 0
    assert not getattr(m.layers[0].attention.qkv, "_int8_quantized", False)
    assert getattr(m.layers[1].attention.qkv, "_int8_quantized", False)
    x, t, fm, fc = _inputs(2, 8, 8, 16, dim, seed=7)
    with torch.no_grad():
        y = m(x.cuda(), t.cuda(), fm.cuda()).cpu()
    assert torch.isfinite(y.float()).all()
    assert "_zib_cache" in m.layers[1].__dict__ and "_zib_cache" not in m.layers[0].__dict__
