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
