"""Benchmark: Z-Image S3-DiT DiT step on B200 through the sm_100a W8A8 path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one forward of the 30-layer S3-DiT block stack (dim 3840, 30 heads
x 128, SwiGLU 10240, adaLN from a 256-d timestep embedding) over one image's
CFG pair at 1024x1024: B=2 rows x (4096 image tokens + 512 text tokens), every
block linear W8A8 + block-Hadamard-128 (the all-linears policy), SDPA over 4608
tokens in bf16.  Random-init weights, seeded N(0,1) synthetic inputs (no
checkpoints or datasets exist offline).  The weights (5.4 GB int8) are far
larger than L2, so each step streams them from HBM; no L2 flush is needed.

With N GPUs (torchrun, one process per GPU, NCCL) each rank runs its own
image (weak scaling) and the final hidden states' latent slice is gathered to
every rank with one NCCL all_gather inside the timed region.

`value` is the whole-job time per DiT step: max-over-ranks elapsed / (K * N).
`--impl reference` times the CPU restatement of the reference path (the
oracle: reference W8A8 arithmetic incl. its bf16-matmul rotation, torch._int_mm
on CPU, CPU SDPA) on a bounded sample and extrapolates to the same unit.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "comfyui-zimage-triton_b200"))

METRIC = "DiT step ms at 1024² (6B, W8A8); INT8 GEMM TOPS and % of peak"
DIM, HEADS, FFN, LAYERS, ADALN = 3840, 30, 10240, 30, 256
GRID, N_TXT, B_CFG = 64, 512, 2
SEQ = GRID * GRID + N_TXT
INT8_DATASHEET_TOPS = 4500.0  # B200 dense INT8, datasheet (the measured peaks hold bf16 and HBM only)
HBM_FALLBACK_GBS = 6650.0  # STREAM-style copy measured earlier on this hardware, used without MEASURED_PEAKS.json
# DRAM bytes (read + write) per launch of each GEMM entry point at the step shapes, from
# one ncu capture (profiles/gemm_w8a8_epilogues_9216rows.md)
NCU_TRAFFIC = {"zib_gemm_w8a8_swiglu_had": 290857216, "zib_gemm_w8a8_swiglu_had_w13": 290541312,
               "zib_gemm_w8a8_qk_norm_rope": 287255040}
NCU_TRAFFIC_SOURCE = "ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/gemm_w8a8_epilogues_9216rows.md"
WORKLOAD = ("30-layer S3-DiT step at 1024x1024 (4096 image + 512 text tokens), CFG pair B=2, "
            "all linears W8A8+Hadamard128, bf16 SDPA")


def _int_ops_per_step(B=B_CFG, S=SEQ):
    M = B * S
    per_block = 2 * M * (DIM * 3 * DIM + DIM * DIM + DIM * 2 * FFN + FFN * DIM)
    return per_block * LAYERS


def _peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {}


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1].split()[0]))
                mx.append(float(parts[2].split()[0]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "samples": len(sm), "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# reference arm / CPU baseline: the oracle on host cores
# ---------------------------------------------------------------------------

def cpu_sample_ms_per_step(rows: int = 64, reps: int = 3) -> tuple[float, dict]:
    """Time one block of the reference's CPU path on `rows` of the B*S token rows and
    extrapolate to a 30-layer step: t * (B*S/rows) * 30.

    Linears use the reference arithmetic (bf16-matmul Hadamard rotation, per-token
    quantisation, torch._int_mm, bf16 dequant epilogue; int8_linear.py:114-138) with
    random int8 weights (timing does not depend on their values); row ops follow
    the Triton kernels' restatement; attention is fp32 CPU SDPA of `rows` queries
    against all 4608 keys per head.
    """
    import torch

    sys.path.insert(0, str(ROOT))
    from oracle import ops

    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(0)
    R = rows

    def rw(n, k):
        return torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8), \
            (torch.rand(n, generator=g) * 1e-3).to(torch.bfloat16)

    W = {"qkv": rw(3 * DIM, DIM), "out": rw(DIM, DIM), "w1": rw(FFN, DIM), "w3": rw(FFN, DIM), "w2": rw(DIM, FFN)}
    x = torch.randn(B_CFG, R // B_CFG, DIM, generator=g).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(DIM, generator=g)).to(torch.bfloat16)
    qn = (1 + 0.1 * torch.randn(128, generator=g)).to(torch.bfloat16)
    mod = (0.1 * torch.randn(B_CFG, DIM, generator=g)).to(torch.bfloat16)
    kv = torch.randn(B_CFG, HEADS, SEQ, 128, generator=g)
    fc = ops.rope_freqs_complex(ops.zimage_positions(GRID, GRID, N_TXT))[: R // B_CFG].unsqueeze(0)

    def lin(key, a):
        wq, sw = W[key]
        q, sx, _ = ops.act_quant_had128_matmul(a)
        return ops.dequant_epilogue(ops.gemm_acc_i32(q, wq), sx, sw, None)

    def block():
        a = ops.modulate(ops.rms_norm(x, nw), mod).reshape(R, DIM)
        qkv = lin("qkv", a).reshape(B_CFG, R // B_CFG, 3, HEADS, 128)
        q = ops.fused_qknorm_rope(qkv[:, :, 0], qn, fc)
        ops.fused_qknorm_rope(qkv[:, :, 1], qn, fc)
        o = torch.nn.functional.scaled_dot_product_attention(q.float().transpose(1, 2), kv, kv)
        o = o.transpose(1, 2).reshape(R, DIM).to(torch.bfloat16)
        ao = lin("out", o).reshape(B_CFG, R // B_CFG, DIM)
        x1 = ops.norm_gate_residual(ao, x, mod, nw)
        f = ops.modulate(ops.rms_norm(x1, nw), mod).reshape(R, DIM)
        h = ops.swiglu(lin("w1", f), lin("w3", f))
        fo = lin("w2", h).reshape(B_CFG, R // B_CFG, DIM)
        return ops.norm_gate_residual(fo, x1, mod, nw)

    block()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        block()
        ts.append(time.perf_counter() - t0)
    t = min(ts)
    ms_step = t * 1e3 * (B_CFG * SEQ / R) * LAYERS
    info = {"sample": f"one block on {R} of {B_CFG * SEQ} token rows (attention: {R} queries x {SEQ} keys), "
                      f"best of {reps}, x{B_CFG * SEQ // R} rows x{LAYERS} layers",
            "cores": torch.get_num_threads(), "block_sample_s": round(t, 4)}
    return ms_step, info


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    vals = []
    info = {}
    for _ in range(max(1, args.warmup // 3)):
        cpu_sample_ms_per_step(rows=64, reps=1)
    for _ in range(args.steps):
        v, info = cpu_sample_ms_per_step(rows=64, reps=1)
        vals.append(v)
    value = statistics.median(vals)
    n = max(1, args.gpus)
    print(json.dumps({
        "metric": METRIC, "impl": "reference", "value": round(value / n, 3), "unit": "ms",
        "n_gpus": n, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(value, 3),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "int8/bf16",
        "data": "synthetic", "config": {"workload": WORKLOAD, "global_batch": B_CFG * n, "seq_len": SEQ,
                                        "parallelism": f"cpu, {info.get('cores')} threads"},
        "cpu_baseline": {"value": round(value / n, 3), "unit": "ms", "cores": info.get("cores"), "kind": "port",
                         "sample": info.get("sample")},
        "e2e": {"value": round(value / n, 3), "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def measure_int_mm_tops(dev) -> float | None:
    """cuBLAS int8 (torch._int_mm) 8192^3, best of 10 - a measured INT8 reference point."""
    import torch

    try:
        n = 8192
        a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
        b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
        for _ in range(3):
            torch._int_mm(a, b.t())
        best = 1e9
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch._int_mm(a, b.t())
            e1.record()
            e1.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        return 2 * n ** 3 / (best * 1e-3) / 1e12
    except Exception:
        return None


def build_model(dev, seed=0):
    import torch

    import nodes
    from zimage_b200.nextdit import NextDiT, random_init_

    torch.manual_seed(seed)
    m = NextDiT(n_layers=LAYERS, dim=DIM, n_heads=HEADS, ffn_dim=FFN, adaln_dim=ADALN, device=dev)
    random_init_(m, seed=seed)
    node = nodes.ZImageTritonApply()
    node.int8_min_dim = 0            # all-linears policy (adaLN 256->15360 included)
    node.int8_skip_sensitive = False

    class _MP:
        pass

    mp = _MP()
    mp.model = _MP()
    mp.model.diffusion_model = m
    node.apply_triton(mp, enable_int8=True)
    return m


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from oracle import ops as _ops  # seeded RoPE table only (positions -> cos/sin)
    from zimage_b200 import _lib
    from zimage_b200.patching import patching_comfyui as pc

    int_mm_tops = measure_int_mm_tops(dev) if rank == 0 else None
    t_setup = time.time()
    model = build_model(dev)
    setup_s = time.time() - t_setup

    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    x = torch.randn(B_CFG, SEQ, DIM, generator=g, device=dev).to(torch.bfloat16)
    t_emb = torch.randn(B_CFG, ADALN, generator=g, device=dev).to(torch.bfloat16)
    freqs = _ops.rope_freqs_matrix(_ops.zimage_positions(GRID, GRID, N_TXT)).unsqueeze(0).to(dev)

    def step(inp):
        with torch.no_grad():
            return model(inp, t_emb, freqs)

    from zimage_b200.shard import gather_images

    def gather(out):
        # this rank's image (its CFG pair) -> latent-sized slice; one NCCL all_gather of all images
        lat = out[:, : GRID * GRID, :64].unsqueeze(0).contiguous()
        return gather_images(lat, world)

    for _ in range(args.warmup):
        y = step(x)
    gather(y)
    torch.cuda.synchronize()
    launches0 = _lib.LAUNCHES
    step(x)
    launches_per_step = _lib.LAUNCHES - launches0  # kernel-launching calls of this library per step
    torch.cuda.synchronize()

    cap = None
    if not args.no_graph:
        from zimage_b200.graph import CapturedStep

        # the whole step as one CUDA graph: same kernels, no per-launch host work or gaps
        cap = CapturedStep(lambda xi, ti: model(xi, ti, freqs), x, t_emb)
        eager_step = step

        def step(inp):  # noqa: F811
            return cap(inp, t_emb)

        for _ in range(args.warmup):
            y = step(x)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    clk = ClockSampler(local)
    clk.start()
    time.sleep(0.3)
    gemm_steps = args.steps
    if cap is None:
        pc.GEMM_EVENTS = []
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        y = step(x)
    gather(y)
    e1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed = e0.elapsed_time(e1)
    launches = launches_per_step * args.steps
    clocks = clk.stop()
    if cap is not None:
        # GEMM launch times for the roofline: the same kernels in eager steps right after
        pc.GEMM_EVENTS = []
        gemm_steps = max(1, min(args.steps, 3))
        for _ in range(gemm_steps):
            eager_step(x)
        torch.cuda.synchronize()
    gem = pc.GEMM_EVENTS
    pc.GEMM_EVENTS = None
    gemm_ms = sum(a.elapsed_time(b) for a, b, _, _ in gem)
    gemm_ops = sum(o for _, _, o, _ in gem)
    per_kernel = {}
    for a_, b_, o_, name_ in gem:
        k = per_kernel.setdefault(name_, {"launches": 0, "ms": 0.0, "ops": 0})
        k["launches"] += 1
        k["ms"] += a_.elapsed_time(b_)
        k["ops"] += o_
    dominant = max(per_kernel, key=lambda k: per_kernel[k]["ms"]) if per_kernel else None
    if world > 1:
        t = torch.tensor([elapsed], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())

    # end to end through the public call with host buffers: H2D inputs, forward, D2H output
    xh = x.cpu().pin_memory()
    th = t_emb.cpu().pin_memory()
    yh = torch.empty(B_CFG, SEQ, DIM, dtype=torch.bfloat16).pin_memory()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    yhs = [yh] + [torch.empty_like(yh).pin_memory() for _ in range(min(args.steps, 2) - 1)]
    torch.cuda.synchronize()
    f0.record()
    if cap is not None:
        # host inputs in / outputs out on a copy stream, overlapped with the graph replays
        from zimage_b200.graph import run_steps_overlapped

        run_steps_overlapped(cap, [(xh, th)] * args.steps, [yhs[i % len(yhs)] for i in range(args.steps)])
        yd = cap.static_out
    else:
        for _ in range(args.steps):
            xd = xh.to(dev, non_blocking=True)
            td = th.to(dev, non_blocking=True)
            with torch.no_grad():
                yd = model(xd, td, freqs)
            yh.copy_(yd, non_blocking=True)
    gather(yd)
    f1.record()
    torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    err = _lib.device_error_read_clear()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, info = cpu_sample_ms_per_step(rows=64, reps=3)
        cpu = {"value": round(v, 3), "unit": "ms", "cores": info["cores"], "kind": "port",
               "sample": info["sample"]}

    if rank == 0:
        ms_step = elapsed / args.steps
        dk = per_kernel.get(dominant) if dominant else None
        achieved = dk["ops"] / (dk["ms"] * 1e-3) / 1e12 if dk and dk["ms"] > 0 else None
        gemm_tops = gemm_ops / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None
        kernels = {k: {"launches": v["launches"], "avg_launch_us": round(v["ms"] * 1e3 / v["launches"], 2),
                       "tops": round(v["ops"] / (v["ms"] * 1e-3) / 1e12, 1),
                       "frac": round(v["ops"] / (v["ms"] * 1e-3) / 1e12 / INT8_DATASHEET_TOPS, 4)}
                   for k, v in per_kernel.items()}
        peaks = _peaks()
        rec = {
            "metric": METRIC, "value": round(ms_step / world, 3), "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 3),
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "int8/bf16",
            "data": "synthetic (seeded N(0,1) latents/text tokens, random-init weights)",
            "config": {"workload": WORKLOAD, "global_batch": B_CFG * world, "seq_len": SEQ,
                       "parallelism": f"dp{world} (images)",
                       "cuda_graph": cap is not None,
                       "l2": "no flush: 5.4 GB int8 weights streamed per step >> 126 MB L2"},
            "roofline": {"kernel": f"{dominant} (tcgen05 kind::i8)", "bound": "tensor",
                         "achieved": None if achieved is None else round(achieved, 1),
                         "peak": INT8_DATASHEET_TOPS, "unit": "TOPS",
                         "frac": None if achieved is None else round(achieved / INT8_DATASHEET_TOPS, 4),
                         "peak_source": "B200 datasheet dense INT8 (no measured INT8 peak: "
                                        + ("MEASURED_PEAKS.json has bf16/HBM only)" if peaks
                                           else "MEASURED_PEAKS.json absent)"),
                         "int_mm_measured_tops": None if int_mm_tops is None else round(int_mm_tops, 1),
                         "frac_of_int_mm": None if (achieved is None or not int_mm_tops)
                         else round(achieved / int_mm_tops, 4),
                         "launches": per_kernel[dominant]["launches"] if dominant else 0,
                         "avg_launch_us": kernels[dominant]["avg_launch_us"] if dominant else None,
                         "traffic": NCU_TRAFFIC.get(dominant),
                         "traffic_source": NCU_TRAFFIC_SOURCE,
                         "all_gemms_tops": None if gemm_tops is None else round(gemm_tops, 1),
                         "gemm_share_of_step": round((gemm_ms / gemm_steps) / max(elapsed / args.steps, 1e-9), 4),
                         "gemm_kernels": kernels,
                         "timing": "CUDA events around each GEMM launch" + (
                             "" if cap is None else " in eager steps right after the graph-timed region")},
            "e2e": {"value": round(e2e_ms / args.steps / world, 3), "unit": "ms",
                    "h2d_bytes_per_step": xh.numel() * 2 + th.numel() * 2,
                    "d2h_bytes_per_step": yh.numel() * 2},
            "gpu_launches": launches,
            "clocks": clocks,
            "int_ops_per_step": _int_ops_per_step(),
            "setup_s": round(setup_s, 1),
            "device_error": err,
            "hbm_peak_gbs": peaks.get("hbm_gbs", HBM_FALLBACK_GBS),
            "hbm_peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
        }
        if cpu:
            rec["cpu_baseline"] = cpu
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch the step's kernels eagerly (no CUDA graph)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
