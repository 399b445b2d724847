"""Generate golden fixtures by running the reference implementation on CPU.

Run in a container where the reference checkout exists (read-only):

    python tests/golden/make_golden.py --ref /root/reference

Writes small fixtures next to this script.  The reference itself is never
needed at test time; the committed fixtures pin the oracle and the kernels.

Fixtures
--------
w8a8_hadamard.pt  reference ``apply_int8_quantization(mode="w8a8_hadamard")`` on a
                  Linear(384 -> 256) with and without bias: ``_w_int8``,
                  ``_w_scale`` and forward outputs for an input with outlier
                  channels, an all-zero row (scale clamp) and a huge row.
w8a8_plain.pt     same for ``mode="w8a8"`` and a K that is not a multiple of 128
                  (the Hadamard-skip path).
policy.json       layer names the reference quantises and its stats dict on a
                  Z-Image-named module tree (reference policy, min_dim=0).
patch_stats.json  stats of the reference ``apply_triton_kernels_comfyui`` on the
                  same tree (a stub ``comfy`` module satisfies its import).
triton_interp.pt  reference Triton kernels run by the Triton interpreter where it
                  works (fp32 swiglu and rope_3d).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import types
from pathlib import Path

# The Triton interpreter must be selected before triton is first imported.
os.environ.setdefault("TRITON_INTERPRET", "1")

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _tree(torch, nn):
    sys.path.insert(0, str(REPO / "comfyui-zimage-triton_b200"))
    from zimage_b200.nextdit import NextDiT

    class ZTree(nn.Module):
        def __init__(self):
            super().__init__()
            d = 128
            self.x_embedder = nn.Linear(64, d)
            self.t_embedder = nn.Sequential(nn.Linear(256, 256), nn.SiLU(), nn.Linear(256, 256))
            self.cap_embedder = nn.Sequential(nn.LayerNorm(256), nn.Linear(256, d))
            m = NextDiT(n_layers=6, dim=d, n_heads=1, ffn_dim=256, adaln_dim=256, dtype=torch.float32)
            self.layers = m.layers
            self.noise_refiner = NextDiT(n_layers=2, dim=d, n_heads=1, ffn_dim=256, dtype=torch.float32).layers
            self.context_refiner = NextDiT(n_layers=2, dim=d, n_heads=1, ffn_dim=256, dtype=torch.float32).layers
            self.final_layer = nn.Sequential(nn.Linear(d, 64))

    torch.manual_seed(0)
    return ZTree()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.ref) / "src"))

    import torch
    import torch.nn as nn
    from zimage_triton.quantization import int8_linear as ref_q

    g = torch.Generator().manual_seed(1234)

    def make_x(M, K):
        x = torch.randn(M, K, generator=g)
        idx = torch.randperm(K, generator=g)[: max(1, K // 100)]
        x[:, idx] *= 20.0
        x[3] = 0.0            # all-zero row -> scale clamp (1e-5)
        x[5] *= 1e4           # huge row
        x[7, :8] = 3e4        # saturating values
        return x.to(torch.bfloat16)

    def run_linear(mode, K, N, bias):
        lin = nn.Linear(K, N, bias=bias)
        with torch.no_grad():
            lin.weight.copy_(torch.randn(N, K, generator=g) * 0.02)
            if bias:
                lin.bias.copy_(torch.randn(N, generator=g) * 0.5)
        lin = lin.to(torch.bfloat16)
        w = lin.weight.detach().clone()
        b = lin.bias.detach().clone() if bias else None
        holder = nn.Module()
        holder.proj = lin
        ref_q._LAST_BLOCKS_RE = None
        stats = ref_q.apply_int8_quantization(holder, min_dim=0, mode=mode)
        x = make_x(48, K)
        with torch.no_grad():
            y = holder.proj(x)
        return {"w": w, "b": b, "x": x, "w_int8": holder.proj._w_int8.clone(),
                "w_scale": holder.proj._w_scale.clone(), "y": y, "stats": stats}

    out = {"bias": run_linear("w8a8_hadamard", 384, 256, True),
           "nobias": run_linear("w8a8_hadamard", 384, 256, False)}
    torch.save(out, HERE / "w8a8_hadamard.pt")
    torch.save({"plain": run_linear("w8a8", 176, 64, False)}, HERE / "w8a8_plain.pt")

    # layer-selection policy
    tree = _tree(torch, nn)
    ref_q._LAST_BLOCKS_RE = None
    st = ref_q.apply_int8_quantization(tree, min_dim=0, mode="w8a8_hadamard")
    names = sorted(n for n, m in tree.named_modules() if getattr(m, "_int8_quantized", False))
    (HERE / "policy.json").write_text(json.dumps({"stats": st, "quantized": names}, indent=1) + "\n")

    # patching stats (stub `comfy` import used by the attention patch)
    comfy = types.ModuleType("comfy")
    ldm = types.ModuleType("comfy.ldm")
    mods = types.ModuleType("comfy.ldm.modules")
    att = types.ModuleType("comfy.ldm.modules.attention")
    att.optimized_attention_masked = lambda *a, **k: None
    sys.modules.update({"comfy": comfy, "comfy.ldm": ldm, "comfy.ldm.modules": mods,
                        "comfy.ldm.modules.attention": att})
    from zimage_triton.models.patching_comfyui import apply_triton_kernels_comfyui

    tree2 = _tree(torch, nn)
    pst = apply_triton_kernels_comfyui(tree2, enable_fused_adaln=False)
    (HERE / "patch_stats.json").write_text(json.dumps(pst, indent=1) + "\n")

    # Triton interpreter (fp32 only; bf16 and libdevice kernels do not run there)
    interp = {}
    try:
        from zimage_triton.kernels.swiglu import triton_swiglu_forward
        gate = torch.randn(8, 320, generator=g)
        up = torch.randn(8, 320, generator=g)
        interp["swiglu"] = {"gate": gate, "up": up, "out": triton_swiglu_forward(gate, up)}
    except Exception as e:  # pragma: no cover - environment dependent
        interp["swiglu_error"] = repr(e)
    try:
        from zimage_triton.kernels.rope_3d import triton_rope_3d
        x = torch.randn(2, 6, 3, 16, generator=g)
        ang = torch.randn(1, 6, 8, generator=g)
        fc = torch.complex(torch.cos(ang), torch.sin(ang))
        interp["rope_3d"] = {"x": x.clone(), "freqs": fc, "out": triton_rope_3d(x.clone(), fc)}
    except Exception as e:  # pragma: no cover
        interp["rope_error"] = repr(e)
    torch.save(interp, HERE / "triton_interp.pt")
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
