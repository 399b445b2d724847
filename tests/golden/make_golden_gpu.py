"""Generate fixtures by running the reference's own code on a B200 GPU (TEST INFRASTRUCTURE).

    python tests/golden/make_golden_gpu.py --ref <dir> [--out DIR] [--only NAME ...]

``<dir>`` holds the reference's ``zimage_triton`` package: its ``src/``
directory, or a ``pip install --target`` of the reference (which is how the
package reaches a GPU machine that has no reference checkout).  The script
runs, on ``cuda:0`` and through the reference's public functions only:

* its Triton kernels (``triton_rms_norm``, ``triton_fused_qknorm_rope``,
  ``triton_fused_norm_gate_residual``, ``triton_swiglu_forward``,
  ``triton_adaln_modulation``, ``triton_rope_3d``) on the seeded inputs of
  ``cases.OPS``, at small shapes and at the benchmark shapes
  ([2, 4608, 30, 128] Q/K, [9216, 3840] norms, [4608, 10240] SwiGLU);
* its W8A8 + Hadamard linear (``apply_int8_quantization(..., "w8a8_hadamard")``
  then ``lin(x)``, torch._int_mm on cuBLASLt) on the small CPU-fixture inputs
  and on the [1024, 3840] -> 11520 QKV linear, recording the int8 activations
  and int32 accumulators it hands to ``torch._int_mm``;
* its patched NextDiT forward, with the node's flags (``nodes.py:151-156``:
  fused norm, SwiGLU, fused QK-norm + RoPE, fused norm+gate+residual; adaLN
  eager) followed by its INT8 quantisation, on a ComfyUI-named module tree
  (one full-width block at 2 x 4608 tokens; 30 layers under the all-linears
  policy and under the node's default policy).  ComfyUI's attention
  dispatcher is replaced by torch SDPA in bf16, which is what it resolves to.

Outputs go to ``ref_gpu_ops.pt``, ``ref_gpu_w8a8.pt`` and ``ref_gpu_models.pt``
(sampled rows of large outputs plus SHA-256 of every input).  The tests read
these files; nothing at test time needs the reference or this script.
"""

from __future__ import annotations

import argparse
import sys
import time
import types
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def _stub_comfy(torch):
    """comfy.ldm.modules.attention.optimized_attention_masked as torch SDPA (ComfyUI's pytorch path):
    q, k, v [B, H, S, d] with skip_reshape=True -> [B, S, H*d]."""
    import torch.nn.functional as F

    def optimized_attention_masked(q, k, v, heads, mask=None, attn_precision=None, skip_reshape=False,
                                   skip_output_reshape=False, transformer_options={}):
        if not skip_reshape:
            b, s, hd = q.shape
            q, k, v = (t.view(b, -1, heads, hd // heads).transpose(1, 2) for t in (q, k, v))
        if mask is not None:
            if mask.dim() == 2:
                mask = mask[:, None, None, :]
            elif mask.dim() == 3:
                mask = mask[:, None]
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask)
        b, h, s, d = o.shape
        return o.transpose(1, 2).reshape(b, s, h * d)

    mods = {n: types.ModuleType(n) for n in ("comfy", "comfy.ldm", "comfy.ldm.modules",
                                             "comfy.ldm.modules.attention")}
    mods["comfy.ldm.modules.attention"].optimized_attention_masked = optimized_attention_masked
    sys.modules.update(mods)


def run_ops(torch, cases, only):
    from zimage_triton.kernels import (triton_adaln_modulation, triton_fused_norm_gate_residual,
                                       triton_fused_qknorm_rope, triton_rms_norm, triton_rope_3d,
                                       triton_swiglu_forward)

    out = {}
    for name, spec in cases.OPS.items():
        if only and name not in only:
            continue
        d = cases.op_inputs(name)
        dv = {k: (v.cuda() if torch.is_tensor(v) else v) for k, v in d.items()}
        k = spec["kind"]
        with torch.no_grad():
            if k == "rms_norm":
                y = triton_rms_norm(dv["x"], dv["weight"], dv["eps"])
            elif k == "qknorm":
                y = triton_fused_qknorm_rope(dv["x"], dv["weight"], dv["freqs_cis"], eps=dv["eps"])
                assert torch.equal(dv["x"].cpu(), d["x"]), "the reference op must leave its input untouched"
            elif k == "ngr":
                y = triton_fused_norm_gate_residual(dv["x"], dv["residual"], dv["gate"], dv["weight"], dv["eps"])
            elif k == "swiglu":
                y = triton_swiglu_forward(dv["gate"], dv["up"])
            elif k == "adaln":
                y = torch.stack(triton_adaln_modulation(dv["raw"], dv["dim"]), 0)  # [4, B, D]
            elif k == "rope":
                y = triton_rope_3d(dv["x"].clone(), dv["freqs_cis"])
        torch.cuda.synchronize()
        flat = y.reshape(-1, y.shape[-1]).cpu()
        rows = cases.op_rows(name, flat.shape[0])
        out[name] = {"in_sha": {kk: cases.sha(v) for kk, v in d.items() if torch.is_tensor(v)},
                     "rows": rows, "out": flat[rows].clone(), "shape": tuple(y.shape)}
        print(f"ops {name}: {tuple(y.shape)} kept {len(rows)} rows", flush=True)
    return out


class _IntMMRecorder:
    """Wraps torch._int_mm to keep the (int8 activations, int32 result) of each call."""

    def __init__(self, torch):
        self.torch = torch
        self.calls = []

    def __enter__(self):
        self.orig = self.torch._int_mm

        def rec(a, b):
            y = self.orig(a, b)
            self.calls.append((a.detach().clone(), y.detach().clone()))
            return y

        self.torch._int_mm = rec
        return self

    def __exit__(self, *exc):
        self.torch._int_mm = self.orig


def run_w8a8(torch, cases, only):
    import torch.nn as nn
    from zimage_triton.quantization import int8_linear as ref_q

    def run(w, b, x, mode):
        N, K = w.shape
        holder = nn.Module()
        holder.proj = nn.Linear(K, N, bias=b is not None, device="cuda", dtype=torch.bfloat16)
        with torch.no_grad():
            holder.proj.weight.copy_(w)
            if b is not None:
                holder.proj.bias.copy_(b)
        ref_q._LAST_BLOCKS_RE = None
        stats = ref_q.apply_int8_quantization(holder, min_dim=0, mode=mode)
        with _IntMMRecorder(torch) as r, torch.no_grad():
            y = holder.proj(x.cuda())
        torch.cuda.synchronize()
        (xq, acc), = r.calls
        return holder.proj._w_int8.cpu(), holder.proj._w_scale.cpu(), xq.cpu(), acc.cpu(), y.cpu(), stats

    out = {}
    small = torch.load(HERE / "w8a8_hadamard.pt")
    for case in ("bias", "nobias"):
        if only and f"small_{case}" not in only:
            continue
        d = small[case]
        wq, ws, xq, acc, y, st = run(d["w"], d["b"], d["x"], "w8a8_hadamard")
        out[f"small_{case}"] = {"in_sha": {"x": cases.sha(d["x"]), "w": cases.sha(d["w"])},
                                "w_int8": wq, "w_scale": ws, "x_int8": xq, "acc": acc, "y": y, "stats": st}
    if not only or "adaln_rows2" in only:
        # the adaLN linear (256 -> 15360) at batch 2: the activation handed to torch._int_mm has 2 rows
        g = torch.Generator().manual_seed(5)
        w = (torch.randn(15360, 256, generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn(2, 256, generator=g).to(torch.bfloat16)
        try:
            run(w, None, x, "w8a8_hadamard")
            out["adaln_rows2"] = {"ok": True}
        except Exception as e:  # recorded: the reference cannot quantise adaLN at batch 2 on a GPU
            out["adaln_rows2"] = {"ok": False, "error": f"{type(e).__name__}: {e}"[:400]}
        print("w8a8 adaln_rows2:", out["adaln_rows2"], flush=True)
    if not only or "cfg1" in only:
        x, w, b = cases.cfg1_linear()
        t0 = time.time()
        wq, ws, xq, acc, y, st = run(w, b, x, "w8a8_hadamard")
        rows = cases.sample_rows(x.shape[0], cases.CFG1_KEEP)
        cols = cases.sample_rows(w.shape[0], cases.CFG1_COLS)
        out["cfg1"] = {"in_sha": {"x": cases.sha(x), "w": cases.sha(w)}, "rows": rows, "cols": cols,
                       "w_int8_sha": cases.sha(wq), "w_scale": ws, "x_int8_sha": cases.sha(xq),
                       "x_int8": xq[rows].clone(), "acc": acc[rows[:8]].clone(), "y": y[rows].clone(),
                       "w_int8_cols": wq[cols].clone(), "acc_cols": acc[rows][:, cols].clone(),
                       "stats": st}
        print(f"w8a8 cfg1 done in {time.time() - t0:.1f}s", flush=True)
    return out


def run_models(torch, cases, only):
    from zimage_triton.models.patching_comfyui import apply_triton_kernels_comfyui
    from zimage_triton.quantization import int8_linear as ref_q

    out = {}
    for name, spec in cases.MODEL.items():
        if only and name not in only:
            continue
        t0 = time.time()
        m = cases.build_model(name, "cuda")
        pstats = apply_triton_kernels_comfyui(m, enable_fused_norm=True, enable_swiglu=True,
                                              enable_fused_qknorm_rope=True, enable_fused_adaln=False,
                                              enable_fused_norm_residual=True)
        ref_q._LAST_BLOCKS_RE = None
        if spec["policy"] == "block_linears":
            orig = ref_q._is_sensitive_layer
            ref_q._is_sensitive_layer = lambda name, n_blocks: False
            try:
                qstats = ref_q.apply_int8_quantization(m, mode="w8a8_hadamard")
            finally:
                ref_q._is_sensitive_layer = orig
        else:
            qstats = ref_q.apply_int8_quantization(m, mode="w8a8_hadamard")
        quantized = sorted(n for n, mod in m.named_modules() if getattr(mod, "_int8_quantized", False))
        x, t, fm = cases.model_inputs(name)
        xd, td, fmd = x.cuda(), t.cuda(), fm.cuda()
        rows = cases.model_rows(name, x.shape[0] * x.shape[1])
        def run(inp):
            kept = {}
            with torch.no_grad():
                h = inp
                for i, layer in enumerate(m.layers):
                    h = layer(h, None, fmd, adaln_input=td)
                    if i in spec["keep_layers"]:
                        kept[i] = h.reshape(-1, h.shape[-1])[rows.cuda()].cpu()
            torch.cuda.synchronize()
            return kept

        kept = run(xd)
        # the same forward on an input moved by one bf16 ulp at a seeded PERTURB_RATE of its
        # values: how far the reference drifts from itself under the smallest input change
        xp = cases.perturb_ulp(x, cases.PERTURB_RATE, seed=spec["xseed"] + 1)
        kept_p = run(xp.cuda())
        out[name] = {"in_sha": {"x": cases.sha(x), "t": cases.sha(t), "freqs": cases.sha(fm)},
                     "rows": rows, "layers": kept, "layers_perturbed": kept_p,
                     "perturbed_values": int((xp != x).sum()), "patch_stats": pstats, "int8_stats": qstats,
                     "quantized": quantized}
        print(f"model {name}: {len(m.layers)} layers, {len(quantized)} int8 linears, "
              f"{time.time() - t0:.1f}s", flush=True)
        del m, xd
        torch.cuda.empty_cache()
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="directory holding the reference's zimage_triton package")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--only", nargs="*", default=[])
    ap.add_argument("--parts", nargs="*", default=["ops", "w8a8", "models"])
    args = ap.parse_args()
    sys.path.insert(0, str(Path(args.ref).resolve()))
    for p in (HERE, REPO / "comfyui-zimage-triton_b200"):
        sys.path.insert(0, str(p))

    import torch

    if not torch.cuda.is_available():
        raise SystemExit("needs a CUDA GPU: the reference's kernels are Triton GPU kernels")
    _stub_comfy(torch)
    import cases
    import triton

    meta = {"torch": str(torch.__version__), "triton": str(triton.__version__),
            "device": torch.cuda.get_device_name(0), "capability": torch.cuda.get_device_capability(0)}
    outd = Path(args.out)
    outd.mkdir(parents=True, exist_ok=True)
    only = set(args.only)
    if "ops" in args.parts:
        torch.save({"meta": meta, "cases": run_ops(torch, cases, only)}, outd / "ref_gpu_ops.pt")
    if "w8a8" in args.parts:
        torch.save({"meta": meta, "cases": run_w8a8(torch, cases, only)}, outd / "ref_gpu_w8a8.pt")
    if "models" in args.parts:
        torch.save({"meta": meta, "cases": run_models(torch, cases, only)}, outd / "ref_gpu_models.pt")
    print("wrote", sorted(p.name for p in outd.glob("ref_gpu_*.pt")), "to", outd, flush=True)


if __name__ == "__main__":
    main()
