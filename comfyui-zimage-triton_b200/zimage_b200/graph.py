"""CUDA-graph replay of a whole DiT step (one capture, then one launch per step).

A 30-layer step issues ~450 kernel launches from Python.  Captured once into a
CUDA graph, a step becomes one graph launch: no per-kernel host work and no
launch gaps between the kernels.  The step must be a pure function of its
tensor inputs (the patched block forward is: no host synchronisation, no
data-dependent host control flow).

Inputs are copied into static buffers before each replay and the output is a
static buffer overwritten by every replay (clone it to keep it).  Tensors that
are not inputs (weights, the RoPE table derived from a fixed ``freqs_cis``)
are baked into the graph: re-capture after changing them, e.g. for a new
resolution.
"""

from __future__ import annotations

from typing import Callable

import torch


class CapturedStep:
    """Capture ``fn(*inputs)`` once; ``__call__`` copies new inputs in and replays."""

    def __init__(self, fn: Callable[..., torch.Tensor], *example_inputs: torch.Tensor, warmup: int = 2):
        if not example_inputs or not all(t.is_cuda for t in example_inputs):
            raise ValueError("CapturedStep needs CUDA tensor inputs")
        self.fn = fn
        self.static_in = [t.detach().clone() for t in example_inputs]
        side = torch.cuda.Stream(device=self.static_in[0].device)
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.no_grad():
            # first calls do one-time host work (device checks, kernel attributes, caches)
            for _ in range(max(1, warmup)):
                fn(*self.static_in)
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.static_out = fn(*self.static_in)

    def __call__(self, *inputs: torch.Tensor) -> torch.Tensor:
        if len(inputs) != len(self.static_in):
            raise ValueError(f"expected {len(self.static_in)} inputs, got {len(inputs)}")
        for dst, src in zip(self.static_in, inputs):
            if src.shape != dst.shape or src.dtype != dst.dtype:
                raise ValueError(f"input {tuple(src.shape)} {src.dtype} does not match the captured "
                                 f"{tuple(dst.shape)} {dst.dtype}; capture a new step")
            if src.data_ptr() != dst.data_ptr():
                dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.static_out

    def replay(self) -> torch.Tensor:
        """Replay on the inputs already in ``static_in``."""
        self.graph.replay()
        return self.static_out


def run_steps_overlapped(cap: CapturedStep, host_inputs: list, host_outputs: list) -> None:
    """Run ``len(host_inputs)`` captured steps with host I/O overlapped with compute.

    Step i reads the pinned host tensors ``host_inputs[i]`` (one per captured input)
    and writes its output into the pinned host tensor ``host_outputs[i]``.  A copy
    stream brings step i+1's inputs into a device staging buffer and drains step
    i-1's output while step i runs on the current stream (double-buffered staging
    on both sides).  On return all copies are enqueued; the current stream is
    ordered after the last one.
    """
    if len(host_inputs) != len(host_outputs):
        raise ValueError("one output buffer per step")
    n = len(host_inputs)
    if n == 0:
        return
    compute = torch.cuda.current_stream()
    copy = torch.cuda.Stream(device=cap.static_out.device)
    dev_in = [[torch.empty_like(t) for t in cap.static_in] for _ in range(2)]
    dev_out = [torch.empty_like(cap.static_out) for _ in range(2)]
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready, in_free, out_ready, out_free = ([ev(), ev()] for _ in range(4))

    def stage_in(i: int) -> None:
        b = i % 2
        with torch.cuda.stream(copy):
            copy.wait_event(in_free[b])  # the buffer's previous step has copied it out
            for d, h in zip(dev_in[b], host_inputs[i]):
                d.copy_(h, non_blocking=True)
            in_ready[b].record(copy)

    stage_in(0)
    for i in range(n):
        b = i % 2
        compute.wait_event(in_ready[b])
        for s, d in zip(cap.static_in, dev_in[b]):
            s.copy_(d, non_blocking=True)
        in_free[b].record(compute)
        if i + 1 < n:
            stage_in(i + 1)
        compute.wait_event(out_free[b])  # step i-2's output has left this buffer
        cap.graph.replay()
        dev_out[b].copy_(cap.static_out, non_blocking=True)
        out_ready[b].record(compute)
        with torch.cuda.stream(copy):
            copy.wait_event(out_ready[b])
            host_outputs[i].copy_(dev_out[b], non_blocking=True)
            out_free[b].record(copy)
    compute.wait_stream(copy)
