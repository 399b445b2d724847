"""Seeded inputs of the reference-on-GPU fixtures (shared by ``make_golden_gpu.py`` and the tests).

Every input is drawn on the CPU from a ``torch.Generator`` with a fixed seed, so
the generator script (run once on a B200 against the reference's own code) and
the tests (run anywhere) build bit-identical inputs; each fixture stores a
SHA-256 of its inputs so a drift in input generation fails loudly instead of
comparing different data.  Model weights of the block and step cases are drawn
on the GPU by ``zimage_b200.nextdit.random_init_`` (seeded Philox), which gives
the same values on every B200 with the same torch build.

Large outputs are stored as sampled rows: row-wise ops (norms, RoPE, SwiGLU,
quantisation) make any subset of rows an exact test of those rows.
"""

from __future__ import annotations

import hashlib

import torch

BF = torch.bfloat16


def sha(t: torch.Tensor) -> str:
    """SHA-256 (first 32 hex digits) of a tensor's bytes."""
    b = t.detach().to("cpu").contiguous().reshape(-1).view(torch.uint8)
    return hashlib.sha256(b.numpy().tobytes()).hexdigest()[:32]


def sample_rows(n: int, k: int) -> torch.Tensor:
    """k row indices spread evenly over [0, n), first and last included."""
    if k >= n:
        return torch.arange(n)
    return torch.unique(torch.linspace(0, n - 1, k).round().long())


def _g(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def norm_weight(n: int, g: torch.Generator) -> torch.Tensor:
    return (1.0 + 0.1 * torch.randn(n, generator=g)).to(BF)


def with_edge_rows(x: torch.Tensor) -> torch.Tensor:
    """Row 1 all zero, row 2 scaled by 1e4, row 3 by 1e-4 (norm and quantiser edge cases)."""
    x = x.clone()
    x[1] = 0
    x[2] = (x[2].float() * 1e4).to(x.dtype)
    x[3] = (x[3].float() * 1e-4).to(x.dtype)
    return x


# ---------------------------------------------------------------------------
# row ops (reference Triton kernels)
# ---------------------------------------------------------------------------

OPS = {
    # name: spec
    "rms_norm_small": dict(kind="rms_norm", rows=40, D=3840, eps=1e-6, seed=101, keep=None),
    "rms_norm_9216": dict(kind="rms_norm", rows=9216, D=3840, eps=1e-5, seed=102, keep=48),
    "rms_norm_head": dict(kind="rms_norm", rows=64, D=128, eps=1e-6, seed=112, keep=None),
    "qknorm_small": dict(kind="qknorm", B=2, gh=8, gw=8, ntxt=16, H=4, eps=1e-6, seed=103, keep=None),
    "qknorm_cfg2_q": dict(kind="qknorm", B=2, gh=64, gw=64, ntxt=512, H=30, eps=1e-6, seed=104, keep=160),
    "qknorm_cfg2_k": dict(kind="qknorm", B=2, gh=64, gw=64, ntxt=512, H=30, eps=1e-6, seed=105, keep=160),
    "ngr_small": dict(kind="ngr", B=2, S=24, D=3840, eps=1e-5, seed=106, keep=None),
    "ngr_9216": dict(kind="ngr", B=2, S=4608, D=3840, eps=1e-5, seed=107, keep=48),
    "swiglu_small": dict(kind="swiglu", rows=6, F=10240, seed=108, keep=None),
    "swiglu_cfg3": dict(kind="swiglu", rows=4608, F=10240, seed=109, keep=24),
    "adaln": dict(kind="adaln", B=2, D=3840, seed=110, keep=None),
    "rope_small": dict(kind="rope", B=2, gh=8, gw=8, ntxt=16, H=4, seed=111, keep=None),
}


def rope_complex(gh: int, gw: int, ntxt: int) -> torch.Tensor:
    """complex64 [1, S, 64] 3-axis table (frame, row, col), axes (32, 48, 48), theta 256."""
    from zimage_b200.nextdit import rope_freqs_complex, zimage_positions

    return rope_freqs_complex(zimage_positions(gh, gw, ntxt)).unsqueeze(0)


def op_inputs(name: str) -> dict:
    """Inputs of one row-op case as CPU tensors (keys as the reference op's arguments)."""
    s = OPS[name]
    g = _g(s["seed"])
    k = s["kind"]
    if k == "rms_norm":
        x = with_edge_rows(torch.randn(s["rows"], s["D"], generator=g).to(BF))
        return {"x": x, "weight": norm_weight(s["D"], g), "eps": s["eps"]}
    if k in ("qknorm", "rope"):
        S = s["gh"] * s["gw"] + s["ntxt"]
        x = torch.randn(s["B"], S, s["H"], 128, generator=g).to(BF)
        d = {"x": x, "freqs_cis": rope_complex(s["gh"], s["gw"], s["ntxt"])}
        if k == "qknorm":
            d["weight"] = norm_weight(128, g)
            d["eps"] = s["eps"]
        return d
    if k == "ngr":
        x = torch.randn(s["B"], s["S"], s["D"], generator=g).to(BF)
        r = torch.randn(s["B"], s["S"], s["D"], generator=g).to(BF)
        gate = (0.5 * torch.randn(s["B"], 1, s["D"], generator=g)).tanh().to(BF)
        x = with_edge_rows(x.reshape(-1, s["D"])).reshape(x.shape)
        return {"x": x, "residual": r, "gate": gate, "weight": norm_weight(s["D"], g), "eps": s["eps"]}
    if k == "swiglu":
        gate = torch.randn(s["rows"], s["F"], generator=g).to(BF)
        up = torch.randn(s["rows"], s["F"], generator=g).to(BF)
        gate[0, :64] = torch.linspace(-90, 90, 64).to(BF)   # saturating SiLU arguments
        return {"gate": gate, "up": up}
    if k == "adaln":
        raw = (0.5 * torch.randn(s["B"], 4 * s["D"], generator=g)).to(BF)
        raw[0, s["D"]:s["D"] + 64] = torch.linspace(-12, 12, 64).to(BF)   # tanh saturation
        return {"raw": raw, "dim": s["D"]}
    raise KeyError(k)


def op_rows(name: str, n_rows: int) -> torch.Tensor:
    keep = OPS[name]["keep"]
    return torch.arange(n_rows) if keep is None else sample_rows(n_rows, keep)


# ---------------------------------------------------------------------------
# W8A8 linear (reference int8_linear.py on the GPU)
# ---------------------------------------------------------------------------

def cfg1_linear(seed_x: int = 0, seed_w: int = 1):
    """W8A8 QKV linear: x bf16 [1024, 3840] ~ N(0,1) with a seeded 1% of channels x20;
    W bf16 [11520, 3840] ~ N(0, 0.02); zero bias."""
    g = _g(seed_x)
    x = torch.randn(1024, 3840, generator=g)
    idx = torch.randperm(3840, generator=g)[:38]
    x[:, idx] *= 20.0
    w = (torch.randn(11520, 3840, generator=_g(seed_w)) * 0.02).to(BF)
    return x.to(BF), w, torch.zeros(11520, dtype=BF)


CFG1_KEEP = 16   # activation rows kept
CFG1_COLS = 64   # output channels whose int8 weights are kept

# ---------------------------------------------------------------------------
# block / step (reference patched forward, ComfyUI-named module tree)
# ---------------------------------------------------------------------------
# Policies: "block_linears" quantises the five linears of every block (qkv, out,
# w1, w3, w2; the first and last blocks included) and keeps adaLN in bf16 - the
# reference cannot quantise adaLN on a GPU at batch 2, because its forward hands
# torch._int_mm a 2-row activation; "reference" is the node's default policy
# (int8_linear.py:27-64: min_dim 1024, sensitive names, first and last two blocks bf16).

MODEL = {
    # name: (n_layers, dim, heads, ffn, grid, n_text, weight seed, input seed, policy, rows kept, layers kept)
    "block_cfg4": dict(L=1, dim=3840, heads=30, ffn=10240, grid=64, ntxt=512, wseed=7, xseed=70,
                       policy="block_linears", keep=48, keep_layers=(0,)),
    "step30_cfg5": dict(L=30, dim=3840, heads=30, ffn=10240, grid=64, ntxt=512, wseed=11, xseed=71,
                        policy="block_linears", keep=16, keep_layers=(0, 4, 9, 19, 29)),
    "step30_default_policy": dict(L=30, dim=3840, heads=30, ffn=10240, grid=64, ntxt=512, wseed=11,
                                  xseed=71, policy="reference", keep=16, keep_layers=(0, 1, 9, 27, 28, 29)),
    "small_default_policy": dict(L=4, dim=1024, heads=8, ffn=2816, grid=8, ntxt=16, wseed=13, xseed=72,
                                 policy="reference", keep=None, keep_layers=(0, 1, 2, 3)),
}


# fraction of input values moved by one bf16 ulp in the reference's self-sensitivity runs: the
# fraction of a block's QKV input that differs between this package and the reference (the
# reference's approximate rsqrt in its RMSNorm), measured on the B200 at 2 x 4608 tokens
PERTURB_RATE = 6e-6


def perturb_ulp(x: torch.Tensor, rate: float, seed: int) -> torch.Tensor:
    """x (bf16) with a seeded `rate` of its values moved to the next bf16 value away from zero."""
    g = torch.Generator().manual_seed(seed)
    pick = torch.rand(x.shape, generator=g) < rate
    bits = x.contiguous().view(torch.int16).clone()
    nz = pick & (x != 0)
    bits[nz] += 1
    return bits.view(torch.bfloat16)


def model_inputs(name: str):
    """(x [B=2, S, dim] bf16, adaln_input [2, 256] bf16, freqs [1, S, 64, 2, 2] fp32) on the CPU."""
    from zimage_b200.nextdit import rope_freqs_matrix, zimage_positions

    s = MODEL[name]
    S = s["grid"] * s["grid"] + s["ntxt"]
    g = _g(s["xseed"])
    x = torch.randn(2, S, s["dim"], generator=g).to(BF)
    t = torch.randn(2, 256, generator=g).to(BF)
    fm = rope_freqs_matrix(zimage_positions(s["grid"], s["grid"], s["ntxt"])).unsqueeze(0)
    return x, t, fm


def build_model(name: str, device):
    """Random-init NextDiT-shaped tree of a model case (weights drawn on `device`)."""
    from zimage_b200.nextdit import NextDiT, random_init_

    s = MODEL[name]
    m = NextDiT(n_layers=s["L"], dim=s["dim"], n_heads=s["heads"], ffn_dim=s["ffn"], device=device)
    random_init_(m, seed=s["wseed"])
    return m


def model_rows(name: str, n_rows: int) -> torch.Tensor:
    keep = MODEL[name]["keep"]
    return torch.arange(n_rows) if keep is None else sample_rows(n_rows, keep)
