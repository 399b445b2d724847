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
    w13 = m.layers[0].__dict__["_zib_cache"]["w13"]
    assert w13 is not None  # w1 and w3 as the halves of one [2F, K] tensor, no second copy
    assert m.layers[0].feed_forward.w1._w_int8.data_ptr() == w13.data_ptr()
    assert torch.equal(y_fused, y_comp)
    # oracle with its own weight prep and fp32 attention: within the attention-numerics band
    p = omodel.prep_layer(params[0], quant_adaln=True)
    want = omodel.block_forward(p, x, fc, t, n_heads=heads)
    assert rel_l2(y_fused.cpu(), want) <= 1.5e-2


def test_fused_block_follows_in_place_weight_updates(cuda):
    """The fused path follows in-place changes of w1 or w3 (the halves of one tensor)."""
    from zimage_b200.patching import patching_comfyui as pc

    dim, heads, ffn = 1024, 8, 2816
    m, _ = _small_model(1, dim, heads, ffn, seed=9)
    _patch(m)
    x, t, fm, _ = _inputs(2, 8, 8, 16, dim, seed=6)
    ff = m.layers[0].feed_forward
    with torch.no_grad():
        y0 = m(x.cuda(), t.cuda(), fm.cuda())
        ff.w1._w_int8[:64].neg_()
        ff.w3._w_int8[-32:].zero_()
        y_fused = m(x.cuda(), t.cuda(), fm.cuda())
        pc.ENABLE_FUSED_BLOCK = False
        try:
            y_comp = m(x.cuda(), t.cuda(), fm.cuda())
        finally:
            pc.ENABLE_FUSED_BLOCK = True
    assert not torch.equal(y_fused, y0)
    assert torch.equal(y_fused, y_comp)


def _record_attention():
    """Wrap the attention call of the patched path; returns (records, restore)."""
    from zimage_b200.patching import patching_comfyui as pc

    rec = []
    orig = pc._attention_bshd

    def wrapped(xq, xk, xv, mask):
        o = orig(xq, xk, xv, mask)
        rec.append(tuple(t.detach().cpu() for t in (xq, xk, xv, o)))
        return o

    pc._attention_bshd = wrapped

    def restore():
        pc._attention_bshd = orig

    return rec, restore


def _replay(rec):
    """Oracle attention that returns the recorded library outputs after checking its inputs."""
    it = iter(rec)

    def attn(q, k, v):
        gq, gk, gv, go = next(it)
        assert torch.equal(q, gq) and torch.equal(k, gk) and torch.equal(v, gv)
        B, S, H, d = q.shape
        return go.reshape(B, S, H * d)

    return attn


def _gpu_weights_into(params, m):
    """Oracle params using the GPU-prepped int8 weights (weight prep is checked bit-exact separately)."""
    out = []
    for blk, p in zip(m.layers, params):
        q = dict(p)
        lins = {"qkv": blk.attention.qkv, "out": blk.attention.out, "w1": blk.feed_forward.w1,
                "w2": blk.feed_forward.w2, "w3": blk.feed_forward.w3, "adaln_w": blk.adaLN_modulation[0]}
        for k, lin in lins.items():
            q[k + "_q"] = lin._w_int8.cpu()
            q[k + "_s"] = lin._w_scale.cpu()
        out.append(q)
    return out


def test_step_bitexact_given_attention_library_outputs(cuda):
    """Full width (dim 3840, 30 heads x 128, FFN 10240), 2 layers, CFG pair: every op of the
    step is bit-exact with the oracle when the oracle is handed the attention library's own
    outputs (and checks it feeds that library bit-identical Q, K, V)."""
    dim, heads, ffn, L = 3840, 30, 10240, 2
    m, params = _small_model(L, dim, heads, ffn, seed=3)
    _patch(m)
    x, t, fm, fc = _inputs(2, 8, 8, 16, dim, seed=8)
    rec, restore = _record_attention()
    try:
        with torch.no_grad():
            y = m(x.cuda(), t.cuda(), fm.cuda()).cpu()
    finally:
        restore()
    assert len(rec) == L
    owq, osw, _ = ops.weight_prep(params[0]["out"])
    assert torch.equal(m.layers[0].attention.out._w_int8.cpu(), owq)
    want = omodel.step_forward(_gpu_weights_into(params, m), x, fc, t, n_heads=heads, attn=_replay(rec))
    assert torch.equal(y, want)
    # the attention library itself, per call, against fp32 attention of the same inputs
    for q, k, v, o in rec:
        ref = ops.sdpa(q, k, v).reshape(o.shape)
        assert rel_l2(o, ref) <= 5e-3
        assert max_abs(o, ref) <= 2e-2


def test_step_follows_in_place_norm_weight_updates(cuda):
    """Full width, 2 layers: the fused norm kernels read the norm modules' current weights.  A
    bf16 weight scaled in place, an fp32 weight holding bf16 values (bf16-weight entry, on a
    copy), then that weight moved off the bf16 grid in place (fp32 entry) each give the oracle's
    bits for the weights of the moment."""
    dim, heads, ffn, L = 3840, 30, 10240, 2
    m, params = _small_model(L, dim, heads, ffn, seed=4)
    _patch(m)
    x, t, fm, fc = _inputs(2, 8, 8, 16, dim, seed=9)
    b0, b1 = m.layers

    def check():
        rec, restore = _record_attention()
        try:
            with torch.no_grad():
                y = m(x.cuda(), t.cuda(), fm.cuda()).cpu()
        finally:
            restore()
        layers = _gpu_weights_into(params, m)
        for blk, q in zip(m.layers, layers):
            for k in ("attention_norm1", "attention_norm2", "ffn_norm1", "ffn_norm2"):
                q[k] = getattr(blk, k).weight.detach().cpu()
        assert torch.equal(y, omodel.step_forward(layers, x, fc, t, n_heads=heads, attn=_replay(rec)))
        return y

    y0 = check()
    with torch.no_grad():
        b1.attention_norm1.weight.mul_(1.25)
    y1 = check()
    assert not torch.equal(y1, y0)
    w = b0.ffn_norm2.weight
    b0.ffn_norm2.weight = torch.nn.Parameter(w.detach().float() * 0.5, requires_grad=False)
    y2 = check()
    assert not torch.equal(y2, y1)
    assert b0.__dict__["_zib_cache"]["fn2_h"] is not None
    with torch.no_grad():
        b0.ffn_norm2.weight.add_(2.0 ** -12)
    y3 = check()
    assert not torch.equal(y3, y2)
    assert b0.__dict__["_zib_cache"]["fn2_h"] is None


def test_step_vs_fp32_attention_oracle(cuda):
    """Against an oracle with fp32 attention the only difference is the attention library's
    bf16 numerics, which the W8A8 re-quantisation of its output amplifies.  Measured:
    rel-L2 ~6e-3 per block, ~1.4e-2 after 3 blocks at this size."""
    dim, heads, ffn, L = 1024, 8, 2816, 3
    m, params = _small_model(L, dim, heads, ffn, seed=1)
    _patch(m)
    x, t, fm, fc = _inputs(2, 8, 8, 16, dim, seed=6)
    rec, restore = _record_attention()
    try:
        with torch.no_grad():
            y = m(x.cuda(), t.cuda(), fm.cuda()).cpu()
    finally:
        restore()
    layers = _gpu_weights_into(params, m)
    assert torch.equal(y, omodel.step_forward(layers, x, fc, t, n_heads=heads, attn=_replay(rec)))
    want = omodel.step_forward(layers, x, fc, t, n_heads=heads)
    assert rel_l2(y, want) <= 3e-2


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


def test_captured_step_replays_the_eager_step(cuda):
    """One CUDA graph per step (zimage_b200.graph.CapturedStep) gives the eager step's bits."""
    from zimage_b200.graph import CapturedStep

    dim, heads, ffn = 1024, 8, 2816
    m, _ = _small_model(2, dim, heads, ffn)
    _patch(m)
    x, t, fm, _ = _inputs(2, 8, 8, 16, dim)
    xd, td, fmd = x.cuda(), t.cuda(), fm.cuda()
    with torch.no_grad():
        want = m(xd, td, fmd).clone()
        x2 = (xd.float() * 0.5).to(torch.bfloat16)
        want2 = m(x2, td, fmd).clone()
    cap = CapturedStep(lambda a, b: m(a, b, fmd), xd, td)
    assert torch.equal(cap(xd, td), want)
    assert torch.equal(cap(x2, td).clone(), want2)   # new inputs are copied in before the replay
    assert torch.equal(cap(x.pin_memory(), t.pin_memory()), want)  # host inputs, copied in
    with pytest.raises(ValueError):
        cap(xd[:1], td)


def test_block_handoff_equals_per_block_path(cuda):
    """The block-final norm fused with the next block's first norm + quantisation is bit-identical."""
    from zimage_b200.patching import patching_comfyui as pc

    dim, heads, ffn = 1024, 8, 2816
    m, _ = _small_model(3, dim, heads, ffn)
    _patch(m)
    assert m.layers[0].__dict__["_zib_next"] is m.layers[1] and m.layers[2].__dict__["_zib_next"] is None
    x, t, fm, _ = _inputs(2, 8, 8, 16, dim)
    with torch.no_grad():
        y_handoff = m(x.cuda(), t.cuda(), fm.cuda())
        assert pc._HANDOFF is None  # consumed by the next block, none left after the last one
        pc.ENABLE_BLOCK_HANDOFF = False
        try:
            y_plain = m(x.cuda(), t.cuda(), fm.cuda())
        finally:
            pc.ENABLE_BLOCK_HANDOFF = True
    assert torch.equal(y_handoff, y_plain)


def test_stacked_adaln_equals_per_block(cuda):
    """One rotation + quantisation + GEMM for every block's adaLN linear gives the per-block
    modulations bit for bit; the blocks' int8 weights become slices of the stack."""
    from zimage_b200.patching import patching_comfyui as pc

    dim, heads, ffn = 1024, 8, 2816
    m, _ = _small_model(3, dim, heads, ffn)
    _patch(m)
    st = m.layers[0].__dict__["_zib_adaln_stack"]
    assert all(b.__dict__["_zib_adaln_stack"] is st for b in m.layers)
    x, t, fm, _ = _inputs(2, 8, 8, 16, dim)
    with torch.no_grad():
        y_stack = m(x.cuda(), t.cuda(), fm.cuda())
        assert st.memo is not None
        first = st.memo[2]
        assert torch.equal(m(x.cuda(), t.cuda(), fm.cuda()), y_stack)
        assert st.memo[2] is not first  # every forward evaluates the stack again
        lin1 = m.layers[1].adaLN_modulation[0]
        assert lin1._w_int8.data_ptr() == st.w.data_ptr() + lin1._w_int8.numel()
        pc.ENABLE_ADALN_STACK = False
        try:
            y_plain = m(x.cuda(), t.cuda(), fm.cuda())
        finally:
            pc.ENABLE_ADALN_STACK = True
    assert torch.equal(y_stack, y_plain)


def test_overlapped_host_io_steps_match_sequential(cuda):
    """run_steps_overlapped (copy stream for host I/O) gives every step's exact output."""
    from zimage_b200.graph import CapturedStep, run_steps_overlapped

    dim, heads, ffn = 1024, 8, 2816
    m, _ = _small_model(1, dim, heads, ffn)
    _patch(m)
    x, t, fm, _ = _inputs(2, 8, 8, 16, dim)
    fmd = fm.cuda()
    xs = [(x * s).to(torch.bfloat16).pin_memory() for s in (1.0, 0.5, -0.25)]
    tp = t.pin_memory()
    with torch.no_grad():
        want = [m(xi.cuda(), t.cuda(), fmd).cpu() for xi in xs]
    cap = CapturedStep(lambda a, b: m(a, b, fmd), xs[0].cuda(), t.cuda())
    outs = [torch.empty_like(w).pin_memory() for w in want]
    run_steps_overlapped(cap, [(xi, tp) for xi in xs], outs)
    torch.cuda.synchronize()
    for o, w in zip(outs, want):
        assert torch.equal(o, w)
