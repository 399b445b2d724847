"""Flow-matching Euler sampling with classifier-free guidance over a batch of images.

The reference's node runs inside ComfyUI, whose KSampler drives the patched
model (``workflows/base/t2i_triton_int8.json``: 30 steps, CFG 4.0, Euler;
``workflows/turbo/t2i_triton_int8.json``: 4 steps, CFG 1.0; both with the
AuraFlow shift 3.0 model sampling).  This module is that loop for the patched
``ZImageDiT`` without ComfyUI:

* schedule: flow time t_i = 1 - i / steps, sigma_i = s t_i / (1 + (s - 1) t_i)
  with shift s (s = 3.0), i = 0 .. steps, so sigma runs from 1 to 0;
* model: velocity v(x, t = 1 - sigma, caption);
* guidance: v = v_uncond + cfg * (v_cond - v_uncond) when cfg != 1 (the
  conditional and unconditional rows run as one batch);
* update: x <- x + (sigma_{i+1} - sigma_i) * v, in fp32.

Images run in fixed micro-batches (two images by default), each step of a
micro-batch captured once as a CUDA graph and replayed.  Every micro-batch has
the same shape whatever the number of GPUs, so an image's latents do not
depend on how the batch is sharded across ranks (``shard.py``).
"""

from __future__ import annotations

import torch

from .graph import CapturedStep


def flow_sigmas(steps: int, shift: float = 3.0) -> torch.Tensor:
    """[steps + 1] fp32 noise levels from 1 to 0 with the time shift s: s t / (1 + (s - 1) t)."""
    if steps < 1:
        raise ValueError(f"steps must be >= 1, got {steps}")
    t = 1.0 - torch.arange(steps + 1, dtype=torch.float64) / steps
    return (shift * t / (1.0 + (shift - 1.0) * t)).float()


class FlowSampler:
    """Euler / CFG sampler of a patched ``ZImageDiT`` over micro-batches of images.

    ``model(x, t, cap)`` maps latents [b, C, H, W] (fp32), flow times [b] and caption
    features [b, L, D] to velocities [b, C, H, W].  With ``cfg != 1`` every step runs the
    conditional and unconditional captions of a micro-batch as one model batch of 2b.
    """

    def __init__(self, model, latent_shape, cap_shape, micro_batch: int = 2, cfg: float = 4.0,
                 steps: int = 30, shift: float = 3.0, device="cuda", use_graph: bool = True):
        self.model = model
        self.b = micro_batch
        self.cfg = float(cfg)
        self.guided = self.cfg != 1.0
        self.steps = steps
        self.sigmas = flow_sigmas(steps, shift)
        self.device = torch.device(device)
        self._sigmas_dev = self.sigmas.to(self.device)
        self.latent_shape = tuple(latent_shape)
        self.cap_shape = tuple(cap_shape)
        rows = 2 * self.b if self.guided else self.b
        self._x = torch.zeros((self.b,) + self.latent_shape, dtype=torch.float32, device=self.device)
        self._cap = torch.zeros((rows,) + self.cap_shape, dtype=torch.bfloat16, device=self.device)
        self._sig = torch.tensor([1.0, 0.9], dtype=torch.float32, device=self.device)
        self.graph = CapturedStep(self._step, self._x, self._cap, self._sig) if use_graph else None

    def _step(self, x: torch.Tensor, cap: torch.Tensor, sig: torch.Tensor) -> torch.Tensor:
        """One Euler step of a micro-batch: x [b, C, H, W] fp32, cap [(2)b, L, D], sig = (sigma, sigma_next)."""
        with torch.no_grad():
            if self.guided:
                xin = torch.cat([x, x], 0)
            else:
                xin = x
            t = (1.0 - sig[0]).expand(xin.shape[0])
            v = self.model(xin, t, cap).float()
            if self.guided:
                vc, vu = v.chunk(2, 0)
                v = vu + self.cfg * (vc - vu)
            return x + (sig[1] - sig[0]) * v

    def captions(self, cond: torch.Tensor, uncond: torch.Tensor | None) -> torch.Tensor:
        """The caption rows of one micro-batch as the model sees them: [cond; uncond] when guided."""
        if self.guided:
            if uncond is None:
                raise ValueError("cfg != 1 needs unconditional caption features")
            return torch.cat([cond, uncond], 0)
        return cond

    def step(self, x: torch.Tensor, cap: torch.Tensor, i: int) -> torch.Tensor:
        """Step i (sigma_i -> sigma_{i+1}) of one micro-batch; returns the new latents (a buffer
        overwritten by the next call when the step is a replayed graph)."""
        sig = self._sigmas_dev[i:i + 2]
        if self.graph is None:
            return self._step(x, cap, sig)
        return self.graph(x, cap, sig)

    def sample(self, latents: torch.Tensor, cond: torch.Tensor, uncond: torch.Tensor | None = None,
               steps: range | None = None) -> torch.Tensor:
        """Run `steps` (default: all) over every micro-batch of `latents` [n, C, H, W]
        (n a multiple of the micro-batch) in place on the device and return them."""
        n = latents.shape[0]
        if n % self.b:
            raise ValueError(f"{n} images do not split into micro-batches of {self.b}")
        caps = [self.captions(cond[j:j + self.b], None if uncond is None else uncond[j:j + self.b])
                for j in range(0, n, self.b)]
        for i in (range(self.steps) if steps is None else steps):
            for k, j in enumerate(range(0, n, self.b)):
                latents[j:j + self.b].copy_(self.step(latents[j:j + self.b], caps[k], i))
        return latents
