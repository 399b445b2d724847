"""LoRA-aware INT8: re-quantising layers whose source weight a LoRA patch changed (GPU).

The reference keeps the INT8 weights of the first load, so LoRA patches written
into quantised layers' (CPU) weights have no effect there (README.md:127-131).
With ``lora_aware`` (node knob ``int8_lora_aware``), ``refresh_int8_weights``
re-quantises exactly the changed layers; results equal a model quantised from
the patched weights in the first place.
"""

import pytest
import torch
import torch.nn as nn

from helpers import seeded_x
from oracle import ops

pytestmark = pytest.mark.gpu


def _low_rank(n, k, r, seed, scale=0.05):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, r, generator=g) @ torch.randn(r, k, generator=g)) * scale


def test_refresh_requantises_a_patched_linear(cuda):
    from zimage_b200 import apply_int8_quantization
    from zimage_b200.quantization import refresh_int8_weights

    g = torch.Generator().manual_seed(0)
    w0 = (torch.randn(256, 384, generator=g) * 0.02).to(torch.bfloat16)
    holder = nn.Module()
    holder.proj = nn.Linear(384, 256, bias=False, dtype=torch.bfloat16, device="cuda")
    with torch.no_grad():
        holder.proj.weight.copy_(w0)
    apply_int8_quantization(holder, min_dim=0, mode="w8a8_hadamard", lora_aware=True)
    lin = holder.proj
    assert holder._int8_lora_aware and refresh_int8_weights(holder) == 0
    # a LoRA delta written into the source weight in place (how a patcher copies a patched weight)
    w1 = (w0.float() + _low_rank(256, 384, 4, seed=1)).to(torch.bfloat16)
    lin.weight.data.copy_(w1)
    assert refresh_int8_weights(holder) == 1 and refresh_int8_weights(holder) == 0
    wq, sw, _ = ops.weight_prep(w1)
    assert torch.equal(lin._w_int8.cpu(), wq) and torch.equal(lin._w_scale.cpu(), sw)
    x = seeded_x(48, 384)
    with torch.no_grad():
        assert torch.equal(lin(x.cuda()).cpu(), ops.w8a8_linear(x, wq, sw, None))
    # removing the patch (a new tensor holding the original weight) re-quantises back
    lin.weight = nn.Parameter(w0.clone(), requires_grad=False)
    assert refresh_int8_weights(holder) == 1
    assert torch.equal(lin._w_int8.cpu(), ops.weight_prep(w0)[0])


@pytest.mark.parametrize("shape,dtype,chunk", [((1000, 333), torch.bfloat16, 4096), ((64, 64), torch.float32, 1 << 20),
                                               ((3, 5, 7), torch.bfloat16, 16)])
def test_source_weights_reach_host_memory_unchanged(cuda, shape, dtype, chunk):
    """apply_int8_quantization moves each quantised layer's source weight to ordinary host memory
    through pinned staging chunks (odd sizes, many chunks, one chunk): the same bits, pageable."""
    from zimage_b200.quantization.int8_linear import _HostMover

    g = torch.Generator().manual_seed(len(shape))
    w = torch.randn(shape, generator=g).to(dtype)
    wd = w.cuda()
    got = _HostMover(chunk_bytes=chunk).move(wd)
    assert got.device.type == "cpu" and not got.is_pinned()
    assert got.dtype == dtype and got.shape == w.shape and torch.equal(got, w)


def _model(params, lora_aware):
    import nodes
    from zimage_b200.nextdit import NextDiT, load_layer_params

    m = NextDiT(n_layers=len(params), dim=1024, n_heads=8, ffn_dim=2816, device="cuda")
    for blk, p in zip(m.layers, params):
        load_layer_params(blk, p)

    class _MP:
        pass

    mp = _MP()
    mp.model = _MP()
    mp.model.diffusion_model = m
    node = nodes.ZImageTritonApply()
    node.int8_min_dim = 0
    node.int8_skip_sensitive = False
    node.int8_lora_aware = lora_aware
    node.apply_triton(mp, enable_int8=True)
    return m


def test_refresh_reaches_the_fused_block_path(cuda):
    """Patched w1 of block 0 and adaLN of block 1 after quantisation: one refresh and the fused
    block path (w1/w3 as halves of one tensor, stacked adaLN) gives the outputs of a model quantised
    from the patched weights."""
    from oracle import model as omodel
    from zimage_b200.quantization import refresh_int8_weights

    gen = torch.Generator().manual_seed(4)
    params = [omodel.make_layer_params(gen, dim=1024, ffn=2816, n_heads=8) for _ in range(2)]
    m = _model(params, lora_aware=True)
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 80, 1024, generator=g).to(torch.bfloat16).cuda()
    t = torch.randn(2, 256, generator=g).to(torch.bfloat16).cuda()
    from zimage_b200.nextdit import rope_freqs_matrix, zimage_positions

    fm = rope_freqs_matrix(zimage_positions(8, 8, 16)).unsqueeze(0).cuda()
    with torch.no_grad():
        y0 = m(x, t, fm).clone()
    patched = [dict(p) for p in params]
    patched[0]["w1"] = (params[0]["w1"].float() + _low_rank(2816, 1024, 8, seed=6)).to(torch.bfloat16)
    patched[1]["adaln_w"] = (params[1]["adaln_w"].float() + _low_rank(4096, 256, 4, seed=7)).to(torch.bfloat16)
    m.layers[0].feed_forward.w1.weight.data.copy_(patched[0]["w1"])
    m.layers[1].adaLN_modulation[0].weight.data.copy_(patched[1]["adaln_w"])
    assert refresh_int8_weights(m) == 2
    fresh = _model(patched, lora_aware=False)
    with torch.no_grad():
        y1 = m(x, t, fm)
        want = fresh(x, t, fm)
    assert not torch.equal(y1, y0)
    assert torch.equal(y1, want)
