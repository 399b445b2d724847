"""Flow-matching sampling (Euler, or the RES second-order multistep method) with
classifier-free guidance over a batch of images.

The reference's node runs inside ComfyUI, whose KSampler drives the patched
model (``workflows/base/t2i_triton_int8.json``: 30 steps, CFG 4.0, sampler
``euler``; ``workflows/turbo/t2i_triton_int8.json``: 4 steps, CFG 1.0, sampler
``res_multistep``; both with scheduler ``simple`` and the AuraFlow shift 3.0
model sampling).  This module is that loop for the patched ``ZImageDiT`` without
ComfyUI:

* schedule ``simple``: the shifted flow noise levels sigma(t) = s t / (1 + (s - 1) t)
  tabulated at t_k = k / 1000 (k = 1 .. 1000, fp32), step j taking entry
  1000 - int(j * 1000 / steps) (the index truncated as a float product), then 0;
  ``linear``: t_j = 1 - j / steps (equal to ``simple`` when steps divides 1000);
* model: velocity v(x, t = 1 - sigma, caption); the denoised estimate is
  D = x - sigma v;
* guidance: v = v_uncond + cfg * (v_cond - v_uncond) when cfg != 1 (the
  conditional and unconditional rows run as one batch);
* ``euler``: x <- x + (sigma' - sigma) v;
* ``res_multistep``: the second-order multistep exponential integrator (RES) of
  Zhang, Song and Chen, "Improved order analysis and design of exponential integrator
  for diffusion models sampling" (arXiv 2308.02157),
  in log-noise time lambda = -log sigma with h = log(sigma / sigma'): the previous
  step's D interpolated linearly in lambda,
  x <- (sigma' / sigma) x + h (b1 D + b2 D_prev), b1 = phi1(-h) - phi2(-h) / r,
  b2 = phi2(-h) / r, r = log(sigma / sigma_prev) / h, phi1(z) = (e^z - 1) / z,
  phi2(z) = (phi1(z) - 1) / z; Euler for the first step and into sigma' = 0.

Every step is x <- a x + b v + c D_prev with host-computed (a, b, c): a = 1,
b = sigma' - sigma, c = 0 for Euler; a = sigma'/sigma + h b1, b = -h b1 sigma,
c = h b2 for the multistep step.  The update runs in fp32.

Images run in fixed micro-batches (two images by default), each step of a
micro-batch captured once as a CUDA graph and replayed; a micro-batch's previous
D stays on the device between its steps.  Every micro-batch has the same shape
whatever the number of GPUs, so an image's latents do not depend on how the
batch is sharded across ranks (``shard.py``).
"""

from __future__ import annotations

import math

import torch

from .graph import CapturedStep

SAMPLERS = ("euler", "res_multistep")
SCHEDULERS = ("simple", "linear")


def flow_sigmas(steps: int, shift: float = 3.0) -> torch.Tensor:
    """``linear`` schedule: [steps + 1] fp32 noise levels s t / (1 + (s - 1) t) at t = 1 - j / steps."""
    if steps < 1:
        raise ValueError(f"steps must be >= 1, got {steps}")
    t = 1.0 - torch.arange(steps + 1, dtype=torch.float64) / steps
    return (shift * t / (1.0 + (shift - 1.0) * t)).float()


def simple_sigmas(steps: int, shift: float = 3.0, table: int = 1000) -> torch.Tensor:
    """``simple`` schedule over the shifted flow table: [steps + 1] fp32 noise levels."""
    if steps < 1:
        raise ValueError(f"steps must be >= 1, got {steps}")
    t = torch.arange(1, table + 1, dtype=torch.float32) / table
    tab = shift * t / (1.0 + (shift - 1.0) * t)
    ss = table / steps
    picks = [float(tab[table - 1 - int(j * ss)]) for j in range(steps)]
    return torch.tensor(picks + [0.0], dtype=torch.float32)


def schedule_sigmas(steps: int, shift: float = 3.0, scheduler: str = "simple") -> torch.Tensor:
    if scheduler == "simple":
        return simple_sigmas(steps, shift)
    if scheduler == "linear":
        return flow_sigmas(steps, shift)
    raise ValueError(f"unknown scheduler {scheduler!r}; one of {SCHEDULERS}")


def step_coefficients(sigmas: torch.Tensor, sampler: str = "euler") -> torch.Tensor:
    """[steps, 4] fp32 rows (sigma_i, a, b, c) of the update x <- a x + b v + c D_prev."""
    if sampler not in SAMPLERS:
        raise ValueError(f"unknown sampler {sampler!r}; one of {SAMPLERS}")
    sg = [float(v) for v in sigmas.double()]
    rows = []
    for i in range(len(sg) - 1):
        s0, s1 = sg[i], sg[i + 1]
        if sampler == "euler" or i == 0 or s1 == 0.0:
            rows.append((s0, 1.0, s1 - s0, 0.0))
            continue
        h = math.log(s0 / s1)
        r = math.log(s0 / sg[i - 1]) / h
        phi1 = math.expm1(-h) / -h
        phi2 = (phi1 - 1.0) / -h
        b1, b2 = phi1 - phi2 / r, phi2 / r
        rows.append((s0, s1 / s0 + h * b1, -h * b1 * s0, h * b2))
    return torch.tensor(rows, dtype=torch.float32)


class FlowSampler:
    """Euler or RES-multistep / CFG sampler of a patched ``ZImageDiT`` over micro-batches of images.

    ``model(x, t, cap)`` maps latents [b, C, H, W] (fp32), flow times [b] and caption
    features [b, L, D] to velocities [b, C, H, W].  With ``cfg != 1`` every step runs the
    conditional and unconditional captions of a micro-batch as one model batch of 2b.
    """

    def __init__(self, model, latent_shape, cap_shape, micro_batch: int = 2, cfg: float = 4.0,
                 steps: int = 30, shift: float = 3.0, device="cuda", use_graph: bool = True,
                 sampler: str = "euler", scheduler: str = "simple"):
        self.model = model
        self.b = micro_batch
        self.cfg = float(cfg)
        self.guided = self.cfg != 1.0
        self.steps = steps
        self.sampler = sampler
        self.sigmas = schedule_sigmas(steps, shift, scheduler)
        self.coefs = step_coefficients(self.sigmas, sampler)
        self.device = torch.device(device)
        self._sigmas_dev = self.sigmas.to(self.device)
        self._coefs_dev = self.coefs.to(self.device)
        self.latent_shape = tuple(latent_shape)
        self.cap_shape = tuple(cap_shape)
        rows = 2 * self.b if self.guided else self.b
        self._zero_d = torch.zeros((self.b,) + self.latent_shape, dtype=torch.float32, device=self.device)
        self._d_prev: dict[int, torch.Tensor] = {}  # micro-batch slot -> its previous step's D
        x = torch.zeros((self.b,) + self.latent_shape, dtype=torch.float32, device=self.device)
        cap = torch.zeros((rows,) + self.cap_shape, dtype=torch.bfloat16, device=self.device)
        self.graph = (CapturedStep(self._step, x, cap, self._coefs_dev[0], self._zero_d) if use_graph else None)

    def _step(self, x: torch.Tensor, cap: torch.Tensor, coef: torch.Tensor, d_prev: torch.Tensor) -> torch.Tensor:
        """One step of a micro-batch: x [b, C, H, W] fp32, cap [(2)b, L, D], coef = (sigma, a, b, c),
        d_prev [b, C, H, W] the previous step's D.  Returns [2, b, C, H, W]: the new x and this D."""
        with torch.no_grad():
            xin = torch.cat([x, x], 0) if self.guided else x
            sigma = coef[0]
            t = (1.0 - sigma).expand(xin.shape[0])
            v = self.model(xin, t, cap).float()
            if self.guided:
                vc, vu = v.chunk(2, 0)
                v = vu + self.cfg * (vc - vu)
            d = x - sigma * v
            return torch.stack([coef[1] * x + coef[2] * v + coef[3] * d_prev, d])

    def eager_step(self, x: torch.Tensor, cap: torch.Tensor, i: int, mb: int = 0) -> torch.Tensor:
        """Step i of micro-batch slot ``mb`` without the graph (the same arithmetic)."""
        out = self._step(x, cap, self._coefs_dev[i], self._d_prev.get(mb, self._zero_d))
        return self._keep(out, mb)

    def _keep(self, out: torch.Tensor, mb: int) -> torch.Tensor:
        if self.sampler != "euler":
            d = self._d_prev.get(mb)
            if d is None:
                d = self._d_prev[mb] = torch.empty_like(self._zero_d)
            d.copy_(out[1])
        return out[0]

    def captions(self, cond: torch.Tensor, uncond: torch.Tensor | None) -> torch.Tensor:
        """The caption rows of one micro-batch as the model sees them: [cond; uncond] when guided."""
        if self.guided:
            if uncond is None:
                raise ValueError("cfg != 1 needs unconditional caption features")
            return torch.cat([cond, uncond], 0)
        return cond

    def step(self, x: torch.Tensor, cap: torch.Tensor, i: int, mb: int = 0) -> torch.Tensor:
        """Step i (sigma_i -> sigma_{i+1}) of the micro-batch in slot ``mb`` (whose previous D the
        multistep sampler keeps); returns the new latents (a buffer overwritten by the next call
        when the step is a replayed graph)."""
        if self.graph is None:
            return self.eager_step(x, cap, i, mb)
        out = self.graph(x, cap, self._coefs_dev[i], self._d_prev.get(mb, self._zero_d))
        return self._keep(out, mb)

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
                latents[j:j + self.b].copy_(self.step(latents[j:j + self.b], caps[k], i, mb=k))
        return latents
