"""Per-kernel microbenchmark of the sm_100a kernels at the Z-Image shapes.

    python -m zimage_b200.kernel_bench [--only a,b] [--iters 20] [--out file.jsonl]

Each kernel runs at the shape it has in the 1024x1024 CFG-pair step (B*S = 9216
token rows, D = 3840, F = 10240, 30 heads x 128) unless noted.  Every timed
iteration is preceded by a 256 MB memset that evicts L2, and is timed alone
with CUDA events on the launch stream; the median is reported.  Bandwidth
kernels report algorithmic bytes / time against the measured HBM copy
bandwidth; GEMMs report 2*M*N*K / time against the dense INT8 datasheet peak.
"""

from __future__ import annotations

import argparse
import json
import statistics
from pathlib import Path

import torch

from . import _lib

HBM_FALLBACK_GBS = 6650.0
INT8_DATASHEET_TOPS = 4500.0
M_TOK, D, F, H, HD, S, B = 9216, 3840, 10240, 30, 128, 4608, 2


def _hbm_peak() -> tuple[float, str]:
    for p in (Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json",):
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json)"
        except Exception:
            pass
    return HBM_FALLBACK_GBS, "fallback"


def _bf16(*shape, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(*shape, generator=g, device="cuda").to(torch.bfloat16)


def _i8(*shape, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randint(-127, 128, shape, generator=g, device="cuda", dtype=torch.int8)


def _empty(*shape, dtype=torch.bfloat16):
    return torch.empty(*shape, dtype=dtype, device="cuda")


def case_act_quant(M=M_TOK, K=D, had=1):
    x, q, sx = _bf16(M, K), _empty(M, K, dtype=torch.int8), _empty(M)
    st = _lib.stream_of(x)

    def run():
        _lib.call("zib_act_quant", x.data_ptr(), K, q.data_ptr(), K, sx.data_ptr(), None, M, K, had, st)

    return run, M * K * 2 + M * K + M * 2, f"[{M},{K}] bf16 -> {'rot128 -> ' if had else ''}int8"


def case_rmsnorm_mod_quant(M=M_TOK, Dm=D):
    x, w, raw = _bf16(M, Dm), torch.ones(Dm, device="cuda"), _bf16(B, 4 * Dm, seed=1) * 0.1
    q, sx = _empty(M, Dm, dtype=torch.int8), _empty(M)
    st = _lib.stream_of(x)

    def run():
        _lib.call("zib_rmsnorm_mod_quant", x.data_ptr(), Dm, w.data_ptr(), raw.data_ptr(), None, 4 * Dm, M // B,
                  q.data_ptr(), Dm, sx.data_ptr(), M, Dm, 1e-5, 1, st)

    return run, M * Dm * 2 + M * Dm + M * 2 + Dm * 4 + B * Dm * 2, f"[{M},{Dm}] norm*mod -> int8"


def case_norm_gate_residual_mod_quant(M=M_TOK, Dm=D, w16=False):
    """w16: the entry with bf16 norm weights (the fused block path's, for bf16 modules)."""
    x, r = _bf16(M, Dm), _bf16(M, Dm, seed=1)
    gates, raw = _bf16(B, 2, Dm, seed=2) * 0.3, _bf16(B, 4 * Dm, seed=3) * 0.1
    w = torch.ones(Dm, device="cuda", dtype=torch.bfloat16 if w16 else torch.float32)
    y, q, sx = _empty(M, Dm), _empty(M, Dm, dtype=torch.int8), _empty(M)
    st = _lib.stream_of(x)
    entry = "zib_norm_gate_residual_mod_quant_w16" if w16 else "zib_norm_gate_residual_mod_quant"

    def run():
        _lib.call(entry, x.data_ptr(), Dm, r.data_ptr(), Dm, gates.data_ptr(), 2 * Dm,
                  M // B, w.data_ptr(), y.data_ptr(), Dm, w.data_ptr(), raw.data_ptr(), None, 4 * Dm, q.data_ptr(),
                  Dm, sx.data_ptr(), M, Dm, 1e-5, 1e-5, 1, st)

    wbytes = 2 * Dm * w.element_size()
    return (run, 3 * M * Dm * 2 + M * Dm + M * 2 + wbytes + 2 * B * Dm * 2,
            f"[{M},{Dm}] x,r -> y + int8" + (" (bf16 norm weights)" if w16 else ""))


def case_norm_gate_residual(M=M_TOK, Dm=D):
    x, r, gates = _bf16(M, Dm), _bf16(M, Dm, seed=1), _bf16(B, 2, Dm, seed=2) * 0.3
    w = torch.ones(Dm, device="cuda")
    y = _empty(M, Dm)
    st = _lib.stream_of(x)

    def run():
        _lib.call("zib_norm_gate_residual", x.data_ptr(), Dm, r.data_ptr(), Dm, gates.data_ptr(), 2 * Dm, M // B,
                  w.data_ptr(), y.data_ptr(), Dm, M, Dm, 1e-5, st)

    return run, 3 * M * Dm * 2 + Dm * 4 + B * Dm * 2, f"[{M},{Dm}] x,r -> y"


def case_swiglu_quant(M=M_TOK, Fm=F):
    h, q, sx = _bf16(M, 2 * Fm), _empty(M, Fm, dtype=torch.int8), _empty(M)
    st = _lib.stream_of(h)

    def run():
        _lib.call("zib_swiglu_quant", h.data_ptr(), 2 * Fm, h.data_ptr() + 2 * Fm, 2 * Fm, q.data_ptr(), Fm,
                  sx.data_ptr(), M, Fm, 1, st)

    return run, M * 2 * Fm * 2 + M * Fm + M * 2, f"[{M},2x{Fm}] -> int8"


def case_swiglu(M=S, Fm=F):
    g, u, o = _bf16(M, Fm), _bf16(M, Fm, seed=1), _empty(M, Fm)
    st = _lib.stream_of(g)

    def run():
        _lib.call("zib_swiglu", g.data_ptr(), Fm, u.data_ptr(), Fm, o.data_ptr(), Fm, M, Fm, st)

    return run, 3 * M * Fm * 2, f"[{M},{Fm}] x2 -> bf16"


def case_qknorm_rope():
    qkv = _bf16(B, S, 3, H, HD)
    cos = torch.rand(S, HD // 2, device="cuda")
    sin = torch.rand(S, HD // 2, device="cuda")
    w = torch.ones(HD, device="cuda")
    st = _lib.stream_of(qkv)
    sb, ss, sh = qkv.stride(0), qkv.stride(1), qkv.stride(3)

    def run():
        for part in (0, 1):
            p = qkv.data_ptr() + part * H * HD * 2
            _lib.call("zib_qknorm_rope", p, sb, ss, sh, p, sb, ss, sh, cos.data_ptr(), sin.data_ptr(), 0,
                      w.data_ptr(), B, S, H, HD, 1e-6, st)

    return run, 2 * 2 * B * S * H * HD * 2 + 2 * S * HD * 4, f"Q,K [{B},{S},{H},{HD}] in place (2 launches)"


def case_gemm(M, N, K):
    q, w = _i8(M, K), _i8(N, K, seed=1)
    sx, sw = _bf16(M).abs() * 1e-2, _bf16(N, seed=2).abs() * 1e-3
    y = _empty(M, N)
    st = _lib.stream_of(q)

    def run():
        _lib.call("zib_gemm_w8a8", q.data_ptr(), K, w.data_ptr(), K, sx.data_ptr(), sw.data_ptr(), None,
                  y.data_ptr(), N, M, N, K, st)

    return run, 2 * M * N * K, f"{M}x{N}x{K} int8 -> bf16"


def case_gemm_swiglu(M, F_, K):
    q, w1, w3 = _i8(M, K), _i8(F_, K, seed=1), _i8(F_, K, seed=3)
    sx, s1, s3 = _bf16(M).abs() * 1e-2, _bf16(F_, seed=2).abs() * 1e-3, _bf16(F_, seed=4).abs() * 1e-3
    y = _empty(M, F_)
    st = _lib.stream_of(q)

    def run():
        _lib.call("zib_gemm_w8a8_swiglu_had", q.data_ptr(), K, w1.data_ptr(), w3.data_ptr(), K, sx.data_ptr(),
                  s1.data_ptr(), s3.data_ptr(), y.data_ptr(), F_, M, F_, K, st)

    return run, 2 * M * 2 * F_ * K, f"{M}x(2x{F_})x{K} int8 -> SwiGLU -> rot128 bf16"


def case_gemm_swiglu_w13(M, F_, K):
    q, w13 = _i8(M, K), _i8(2 * F_, K, seed=1)   # [w1; w3]: the two weights as halves of one tensor
    sx, s1, s3 = _bf16(M).abs() * 1e-2, _bf16(F_, seed=2).abs() * 1e-3, _bf16(F_, seed=4).abs() * 1e-3
    st = _lib.stream_of(q)
    y = _empty(M, F_)

    def run():
        _lib.call("zib_gemm_w8a8_swiglu_had_w13", q.data_ptr(), K, w13.data_ptr(), K, sx.data_ptr(),
                  s1.data_ptr(), s3.data_ptr(), y.data_ptr(), F_, M, F_, K, st)

    return run, 2 * M * 2 * F_ * K, f"{M}x(2x{F_})x{K} int8 (w1/w3 halves of one tensor) -> SwiGLU -> rot128 bf16"


def case_gemm_qk_rope(M, K):
    N = 3 * H * HD
    q, w = _i8(M, K), _i8(N, K, seed=1)
    sx, sw = _bf16(M).abs() * 1e-2, _bf16(N, seed=2).abs() * 1e-3
    qn, kn = torch.ones(HD, device="cuda"), torch.ones(HD, device="cuda")
    ang = torch.rand(S, HD // 2, device="cuda")
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    y = _empty(M, N)
    st = _lib.stream_of(q)

    def run():
        _lib.call("zib_gemm_w8a8_qk_norm_rope", q.data_ptr(), K, w.data_ptr(), K, sx.data_ptr(), sw.data_ptr(),
                  y.data_ptr(), N, M, N, K, qn.data_ptr(), kn.data_ptr(), 1e-5, 1e-5, cos.data_ptr(),
                  sin.data_ptr(), 0, S, H, st)

    return run, 2 * M * N * K, f"{M}x{N}x{K} int8 -> QK-norm + RoPE bf16"


def case_weight_prep(N=3 * D, K=D):
    w, wq, sw = _bf16(N, K) * 0.02, _empty(N, K, dtype=torch.int8), _empty(N)
    st = _lib.stream_of(w)

    def run():
        _lib.call("zib_weight_prep", w.data_ptr(), K, wq.data_ptr(), K, sw.data_ptr(), None, None, 0, N, K, 1, st)

    return run, N * K * 2 + N * K + N * 2, f"[{N},{K}] bf16 -> int8 (offline)"


def case_cfg3_ffn_block(M=S, Dm=D, Fm=F):
    """The SwiGLU FFN block at 4608 rows as the fused block path runs it: RMSNorm * (1 + scale)
    -> rotate -> int8; w1/w3 GEMM + SwiGLU + rotation (w1/w3 halves of one tensor); int8 quantise; w2 GEMM."""
    x, w, raw = _bf16(M, Dm), torch.ones(Dm, device="cuda"), _bf16(1, 4 * Dm, seed=1) * 0.1
    w13, w2 = _i8(2 * Fm, Dm, seed=2), _i8(Dm, Fm, seed=3)
    s1, s3, s2 = (torch.rand(n, device="cuda").to(torch.bfloat16) * 1e-3 for n in (Fm, Fm, Dm))
    q, sx = _empty(M, Dm, dtype=torch.int8), _empty(M)
    xr, qh, sxh, out = _empty(M, Fm), _empty(M, Fm, dtype=torch.int8), _empty(M), _empty(M, Dm)
    st = _lib.stream_of(x)

    def run():
        _lib.call("zib_rmsnorm_mod_quant", x.data_ptr(), Dm, w.data_ptr(), raw.data_ptr(), None, 4 * Dm, M,
                  q.data_ptr(), Dm, sx.data_ptr(), M, Dm, 1e-5, 1, st)
        _lib.call("zib_gemm_w8a8_swiglu_had_w13", q.data_ptr(), Dm, w13.data_ptr(), Dm, sx.data_ptr(),
                  s1.data_ptr(), s3.data_ptr(), xr.data_ptr(), Fm, M, Fm, Dm, st)
        _lib.call("zib_act_quant", xr.data_ptr(), Fm, qh.data_ptr(), Fm, sxh.data_ptr(), None, M, Fm, 0, st)
        _lib.call("zib_gemm_w8a8", qh.data_ptr(), Fm, w2.data_ptr(), Fm, sxh.data_ptr(), s2.data_ptr(), None,
                  out.data_ptr(), Dm, M, Dm, Fm, st)

    return run, 2 * M * 2 * Fm * Dm + 2 * M * Fm * Dm, f"[{M},{Dm}] norm*mod->int8, w13+SwiGLU, int8, w2"


def case_sdpa():
    """torch SDPA (library) at the block's shape, for the step's time budget."""
    q = _bf16(B, S, 3, H, HD)
    xq, xk, xv = (q[:, :, i].transpose(1, 2) for i in range(3))

    def run():
        torch.nn.functional.scaled_dot_product_attention(xq, xk, xv)

    return run, 4 * B * H * S * S * HD, f"[{B},{H},{S},{HD}] bf16 (torch SDPA, library)"


CASES = {
    "act_quant": (lambda: case_act_quant(), "hbm"),
    "act_quant_m1024": (lambda: case_act_quant(1024, D), "hbm"),
    "act_quant_k10240": (lambda: case_act_quant(M_TOK, F), "hbm"),
    "act_quant_plain_k10240": (lambda: case_act_quant(M_TOK, F, had=0), "hbm"),
    "rmsnorm_mod_quant": (lambda: case_rmsnorm_mod_quant(), "hbm"),
    "norm_gate_residual_mod_quant": (lambda: case_norm_gate_residual_mod_quant(), "hbm"),
    "norm_gate_residual_mod_quant_w16": (lambda: case_norm_gate_residual_mod_quant(w16=True), "hbm"),
    "norm_gate_residual": (lambda: case_norm_gate_residual(), "hbm"),
    "swiglu_quant": (lambda: case_swiglu_quant(), "hbm"),
    "swiglu": (lambda: case_swiglu(), "hbm"),
    "swiglu_quant_s4608": (lambda: case_swiglu_quant(S, F), "hbm"),
    "cfg3_ffn_block": (lambda: case_cfg3_ffn_block(), "int8"),
    "qknorm_rope": (lambda: case_qknorm_rope(), "hbm"),
    "weight_prep": (lambda: case_weight_prep(), "hbm"),
    "gemm_cfg1_qkv_m1024": (lambda: case_gemm(1024, 3 * D, D), "int8"),
    "gemm_one_tile": (lambda: case_gemm(256, 256, 128), "int8"),  # the launch's fixed cost
    "gemm_adaln_stack": (lambda: case_gemm(2, 30 * 4 * D, 256), "int8"),
    "gemm_qkv": (lambda: case_gemm(M_TOK, 3 * D, D), "int8"),
    "gemm_out": (lambda: case_gemm(M_TOK, D, D), "int8"),
    "gemm_w13": (lambda: case_gemm(M_TOK, 2 * F, D), "int8"),
    "gemm_w2": (lambda: case_gemm(M_TOK, D, F), "int8"),
    "gemm_qkv_qk_rope": (lambda: case_gemm_qk_rope(M_TOK, D), "int8"),
    "gemm_w13_swiglu_had": (lambda: case_gemm_swiglu(M_TOK, F, D), "int8"),
    "gemm_w13_swiglu_had_w13": (lambda: case_gemm_swiglu_w13(M_TOK, F, D), "int8"),
    "gemm_w13_swiglu_had_w13_m18432": (lambda: case_gemm_swiglu_w13(2 * M_TOK, F, D), "int8"),
    "gemm_qkv_qk_rope_m18432": (lambda: case_gemm_qk_rope(2 * M_TOK, D), "int8"),
    "gemm_out_m18432": (lambda: case_gemm(2 * M_TOK, D, D), "int8"),
    "gemm_w2_m18432": (lambda: case_gemm(2 * M_TOK, D, F), "int8"),
    "sdpa_torch": (lambda: case_sdpa(), "bf16"),
}


def run_case(name: str, iters: int, flush: torch.Tensor) -> dict:
    run, work, shape = CASES[name][0]()
    kind = CASES[name][1]
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    evs = []
    for _ in range(iters):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    ts = [a.elapsed_time(b) for a, b in evs]
    med = statistics.median(ts)
    rec = {"kernel": name, "shape": shape, "ms_median": round(med, 4), "ms_min": round(min(ts), 4)}
    if kind == "hbm":
        peak, src = _hbm_peak()
        gbs = work / (med * 1e-3) / 1e9
        rec.update(bytes=work, gbs=round(gbs, 1), peak_gbs=peak, frac=round(gbs / peak, 4), peak_source=src)
    elif kind == "int8":
        tops = work / (med * 1e-3) / 1e12
        rec.update(ops=work, tops=round(tops, 1), peak_tops=INT8_DATASHEET_TOPS,
                   frac=round(tops / INT8_DATASHEET_TOPS, 4), peak_source="datasheet dense INT8")
    else:
        tf = work / (med * 1e-3) / 1e12
        rec.update(flops=work, tflops=round(tf, 1))
    return rec


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--out", default="")
    a = ap.parse_args()
    names = [n for n in a.only.split(",") if n] or list(CASES)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device="cuda")
    lines = []
    for n in names:
        rec = run_case(n, a.iters, flush)
        lines.append(json.dumps(rec))
        print(lines[-1], flush=True)
    err = _lib.device_error_read_clear()
    if err:
        raise RuntimeError(f"device error word set: {err}")
    if a.out:
        Path(a.out).write_text("\n".join(lines) + "\n")


if __name__ == "__main__":
    main()
