"""W8A8 (+ block Hadamard) INT8 linear layers on sm_100a.

Replaces ``src/zimage_triton/quantization/int8_linear.py`` of the reference
with the same module-replacement surface, so ComfyUI glue written against it
keeps working:

* per quantised ``nn.Linear``: buffers ``_w_int8`` (int8 [out, in], weight
  pre-rotated by the block Hadamard when ``in % 128 == 0``) and ``_w_scale``
  (per-output-channel scale in the weight dtype); attributes
  ``_int8_quantized``, ``_int8_use_hadamard``, ``_int8_layer_name``,
  ``_int8_sd_hook``; instance ``forward`` and ``_apply`` overrides; the bf16
  ``weight`` moved to CPU (int8_linear.py:273-308);
* the same layer-selection policy and stats keys (int8_linear.py:27-64,
  :209-321) and the same restore path (int8_linear.py:324-384).

The forward is two kernel launches: ``zib_act_quant`` (rotation + per-token
absmax + int8, int8_linear.py:119-130) and ``zib_gemm_w8a8`` (tcgen05 int8
GEMM with the dequant/bias epilogue fused, int8_linear.py:133-137).  Weight
prep runs on the GPU (``zib_weight_prep``) even when the module sits on the
CPU at patch time; the buffers are then placed on the weight's device.
"""

from __future__ import annotations

import logging
import re
import types

import torch
import torch.nn as nn

from .. import _lib

logger = logging.getLogger(__name__)

_MIN_DIM = 1024
_HADAMARD_GROUP_SIZE = 128  # Z-Image head_dim; 3840/128 = 30, 10240/128 = 80

# Layers kept in the source dtype by the reference policy (int8_linear.py:30-38).
_SENSITIVE_PATTERNS: list[str] = [
    "cap_embedder",
    "t_embedder",
    "x_embedder",
    "adaLN_modulation",
    "context_refiner",
    "noise_refiner",
    "final_layer",
]

_FIRST_BLOCK_RE = re.compile(r"layers\.0\.")


def _is_sensitive_layer(name: str, n_blocks: int) -> bool:
    """int8_linear.py:44-56.  The last-two-blocks pattern is derived from this
    model's block count on every call (the reference caches the first model's)."""
    for pattern in _SENSITIVE_PATTERNS:
        if pattern in name:
            return True
    if _FIRST_BLOCK_RE.search(name):
        return True
    if n_blocks > 2:
        last = "|".join(str(i) for i in range(n_blocks - 2, n_blocks))
        if re.search(rf"layers\.({last})\.", name):
            return True
    return False


def _count_blocks(model: nn.Module) -> int:
    return sum(1 for m in model.modules() if type(m).__name__ == "JointTransformerBlock")


def _prep_device(weight: torch.Tensor) -> torch.device:
    if weight.is_cuda:
        return weight.device
    if not torch.cuda.is_available():
        raise RuntimeError("zimage_b200 INT8 weight prep needs an sm_100 CUDA device; none is visible")
    return torch.device("cuda", torch.cuda.current_device())


def quantize_weight(weight: torch.Tensor, hadamard: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Rotate (optional) + per-channel int8 quantisation on the GPU.

    Returns (w_int8 [out, in] int8, w_scale [out] bf16) on the GPU; the same
    arithmetic as rotate_weight + _quantize_weight_per_channel
    (hadamard.py:47-75, int8_linear.py:67-73), rotation exact then rounded to fp32.
    """
    dev = _prep_device(weight)
    w = weight.detach()
    wb = w.to(device=dev, dtype=torch.bfloat16)
    if w.dtype != torch.bfloat16 and not torch.equal(wb.float(), w.to(dev).float()):
        raise ValueError(f"INT8 weight prep expects bf16-representable weights, got {w.dtype}")
    wb = wb.contiguous()
    N, K = wb.shape
    _lib.require_device(wb)
    wq = torch.empty(N, K, dtype=torch.int8, device=dev)
    sw = torch.empty(N, dtype=torch.bfloat16, device=dev)
    _lib.call("zib_weight_prep", wb.data_ptr(), K, wq.data_ptr(), K, sw.data_ptr(), None, None, 0, N, K,
              1 if hadamard else 0, _lib.stream_of(wb))
    return wq, sw


# --- forward builders --------------------------------------------------------

def w8a8_forward_2d(x2: torch.Tensor, w_int8: torch.Tensor, w_scale: torch.Tensor,
                    bias: torch.Tensor | None, hadamard: bool) -> torch.Tensor:
    """[M, K] bf16 -> [M, N] bf16 through act_quant + tcgen05 GEMM."""
    _lib.require_device(x2)
    if x2.dtype != torch.bfloat16:
        raise ValueError(f"W8A8 forward computes in bfloat16; got {x2.dtype}")
    if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    M, K = x2.shape
    N = w_int8.shape[0]
    stream = _lib.stream_of(x2)
    q = torch.empty(M, K, dtype=torch.int8, device=x2.device)
    sx = torch.empty(M, dtype=torch.bfloat16, device=x2.device)
    _lib.call("zib_act_quant", x2.data_ptr(), x2.stride(0), q.data_ptr(), K, sx.data_ptr(), None, M, K,
              1 if hadamard else 0, stream)
    y = torch.empty(M, N, dtype=torch.bfloat16, device=x2.device)
    fused_bias = bias if (bias is not None and bias.dtype == torch.bfloat16 and bias.is_cuda) else None
    _lib.call("zib_gemm_w8a8", q.data_ptr(), K, w_int8.data_ptr(), w_int8.stride(0), sx.data_ptr(),
              w_scale.data_ptr(), _lib.ptr(fused_bias), y.data_ptr(), N, M, N, K, stream)
    if bias is not None and fused_bias is None:
        y = y + bias
    return y


def _make_w8a8_forward(module: nn.Linear, hadamard: bool):
    """W8A8 forward (int8_linear.py:79-99 / :102-140), kernels on sm_100a."""
    bias = module.bias
    out_f = module.out_features

    def _forward(self, x: torch.Tensor) -> torch.Tensor:
        orig_shape = x.shape
        y = w8a8_forward_2d(x.reshape(-1, orig_shape[-1]), self._w_int8, self._w_scale, bias, hadamard)
        return y.view(*orig_shape[:-1], out_f)

    return types.MethodType(_forward, module)


def _int8_state_dict_hook(module, state_dict, prefix, local_metadata) -> None:
    """Hide the CPU weight from state_dict (int8_linear.py:154-170)."""
    key = prefix + "weight"
    if key in state_dict:
        del state_dict[key]


def _int8_apply(self, fn, recurse=True):
    """Custom _apply (int8_linear.py:173-200): weight stays on CPU; INT8 buffers
    may move to the GPU but never back."""
    if recurse:
        for module in self.children():
            module._apply(fn)
    for key, param in self._parameters.items():
        if param is None or key == "weight":
            continue
        self.register_parameter(key, torch.nn.Parameter(fn(param), requires_grad=False))
    for key, buf in self._buffers.items():
        if buf is not None:
            if key in ("_w_int8", "_w_scale") and buf.device.type == "cuda":
                continue
            self._buffers[key] = fn(buf)
    return self


_VALID_MODES = ("w8a8", "w8a8_hadamard", "w8a16")
_B200_MODES = ("w8a8", "w8a8_hadamard")

# Layer-selection policies:
#   "reference"   - the reference's (int8_linear.py:44-56): sensitive names, layers.0 and the
#                   last two blocks stay in the source dtype;
#   "all_linears" - every nn.Linear with in/out >= min_dim;
#   "main_layers" - every nn.Linear of the main block list ``layers.N.`` (adaLN included, first
#                   and last blocks included); embedders, refiners and the final layer stay in
#                   the source dtype as the reference keeps them.
_POLICIES = ("reference", "all_linears", "main_layers")
_MAIN_LAYER_RE = re.compile(r"^(?:.*\.)?layers\.\d+\.")


def _policy_skips(policy: str, name: str, n_blocks: int) -> bool:
    if policy == "reference":
        return _is_sensitive_layer(name, n_blocks)
    if policy == "main_layers":
        return _MAIN_LAYER_RE.match(name) is None
    return False


def select_layers(model: nn.Module, min_dim: int = _MIN_DIM, mode: str = "w8a8",
                  skip_sensitive: bool = True, policy: str | None = None):
    """Layer-selection policy of apply_int8_quantization (int8_linear.py:242-271), no side effects.

    ``policy`` (one of "reference", "all_linears", "main_layers") overrides
    ``skip_sensitive`` (True = "reference", False = "all_linears").
    Returns ([(name, module, use_hadamard), ...], stats).
    """
    if mode not in _VALID_MODES:
        raise ValueError(f"Unknown mode: {mode!r}. Use one of {_VALID_MODES}")
    if mode not in _B200_MODES:
        # the reference's weight-only mode (int8_linear.py:143-151) dequantises the whole weight
        # and calls F.linear in eager torch on every forward; the node never selects it
        raise ValueError(f"mode {mode!r} (weight-only INT8 through a dequantised bf16 F.linear) is not "
                         f"provided on the sm_100a path; use one of {_B200_MODES}")
    if policy is None:
        policy = "reference" if skip_sensitive else "all_linears"
    if policy not in _POLICIES:
        raise ValueError(f"Unknown policy: {policy!r}. Use one of {_POLICIES}")
    use_hadamard = mode == "w8a8_hadamard"
    n_blocks = _count_blocks(model)
    stats = {"quantized": 0, "skipped": 0, "sensitive": 0, "had_skipped": 0}
    plan = []
    for name, module in list(model.named_modules()):
        if not isinstance(module, nn.Linear):
            continue
        in_f, out_f = module.in_features, module.out_features
        if in_f < min_dim or out_f < min_dim:
            stats["skipped"] += 1
            continue
        if _policy_skips(policy, name, n_blocks):
            stats["sensitive"] += 1
            continue
        if in_f % 16 != 0:
            # the tcgen05 GEMM streams K in 16-byte TMA rows
            stats["skipped"] += 1
            logger.debug("INT8 skip %s: in=%d not a multiple of 16", name, in_f)
            continue
        had = use_hadamard and in_f % _HADAMARD_GROUP_SIZE == 0
        if use_hadamard and not had:
            stats["had_skipped"] += 1
            logger.debug("Hadamard skip %s: in=%d not divisible by %d", name, in_f, _HADAMARD_GROUP_SIZE)
        plan.append((name, module, had))
        stats["quantized"] += 1
    return plan, stats


def weight_fingerprint(w: torch.Tensor) -> tuple:
    """(storage pointer, version counter, hash of 4096 values at fixed strided positions) of a
    weight: a low-rank update such as a LoRA patch changes nearly every value of the weight, so
    it changes the sampled values whether it replaces the tensor or writes into it."""
    flat = w.detach().reshape(-1)
    n = flat.numel()
    k = min(n, 4096)
    idx = (torch.arange(k, dtype=torch.int64) * (n - 1)) // max(k - 1, 1)  # exact integer positions
    idx = idx.to(flat.device)
    return (w.data_ptr(), w._version, hash(flat[idx].float().cpu().numpy().tobytes()))


class _HostMover:
    """Moves CUDA tensors into ordinary (pageable) host memory through two pinned staging
    buffers: each chunk's device-to-host copy runs at pinned-memory speed while the host copies
    the previous chunk out of the other buffer.  A pageable ``.to("cpu")`` goes through the
    driver's own staging and measured 2.0 GB/s on a B200 machine for the 12.3 GB of bf16
    linear weights of the 30-layer model."""

    def __init__(self, chunk_bytes: int = 64 << 20):
        self.chunk = chunk_bytes
        self.stage: list[torch.Tensor] = []
        self.done: list[torch.cuda.Event] = []

    def move(self, t: torch.Tensor) -> torch.Tensor:
        if not t.is_cuda or t.numel() == 0:
            return t.to(device="cpu")
        if not self.stage:
            self.stage = [torch.empty(self.chunk, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
            self.done = [torch.cuda.Event(), torch.cuda.Event()]
        src = t.detach().contiguous().reshape(-1).view(torch.uint8)
        dst = torch.empty(t.shape, dtype=t.dtype, device="cpu")
        out = dst.reshape(-1).view(torch.uint8)
        stream = torch.cuda.current_stream(t.device)
        pending: list[tuple[int, int] | None] = [None, None]
        n, c = src.numel(), self.chunk
        for i, off in enumerate(range(0, n, c)):
            k = i % 2
            if pending[k] is not None:  # the buffer's previous chunk: wait for it, then drain it
                self.done[k].synchronize()
                o, m = pending[k]
                out[o:o + m].copy_(self.stage[k][:m])
            m = min(c, n - off)
            self.stage[k][:m].copy_(src[off:off + m], non_blocking=True)
            self.done[k].record(stream)
            pending[k] = (off, m)
        for k in (0, 1):  # the last chunk of each buffer
            if pending[k] is not None:
                self.done[k].synchronize()
                o, m = pending[k]
                out[o:o + m].copy_(self.stage[k][:m])
        return dst


def apply_int8_quantization(model: nn.Module, min_dim: int = _MIN_DIM, mode: str = "w8a8",
                            skip_sensitive: bool = True, policy: str | None = None,
                            lora_aware: bool = False) -> dict[str, int]:
    """Quantise qualifying nn.Linear layers in place (int8_linear.py:209-321).

    ``skip_sensitive=False`` quantises every linear with in/out >= ``min_dim``
    (the all-linears policy); the default reproduces the reference policy;
    ``policy`` selects one of "reference", "all_linears", "main_layers" by name.
    ``lora_aware=True`` marks the model so that ``refresh_int8_weights`` (which the
    ComfyUI model patcher calls after applying or removing weight patches) re-quantises
    every layer whose source weight changed; the reference keeps the INT8 weights of
    the first load and ignores LoRA on quantised layers (README.md:127-131).
    Returns {"quantized", "skipped", "sensitive", "had_skipped"}.
    """
    plan, stats = select_layers(model, min_dim, mode, skip_sensitive, policy)
    mover = _HostMover()
    for name, module, had in plan:
        in_f, out_f = module.in_features, module.out_features
        w_int8, w_scale = quantize_weight(module.weight.data, had)
        target = module.weight.device
        module.register_buffer("_w_int8", w_int8.to(target))
        module.register_buffer("_w_scale", w_scale.to(device=target, dtype=module.weight.dtype))
        module.weight.data = mover.move(module.weight.data)
        module._int8_src = weight_fingerprint(module.weight)

        module.forward = _make_w8a8_forward(module, had)
        module._int8_quantized = True
        module._int8_use_hadamard = had
        module._int8_layer_name = name
        module._apply = types.MethodType(_int8_apply, module)
        module._int8_sd_hook = module._register_state_dict_hook(_int8_state_dict_hook)
        logger.debug("INT8 [%s] %s (%d->%d)", mode, name, in_f, out_f)

    if lora_aware:
        model._int8_lora_aware = True
    logger.info("INT8 [%s]: %d quantized, %d skipped, %d sensitive, %d had_skip", mode,
                stats["quantized"], stats["skipped"], stats["sensitive"], stats["had_skipped"])
    return stats


def refresh_int8_weights(model: nn.Module) -> int:
    """Re-quantise every INT8 layer whose source weight changed since it was quantised.

    The source weight (on the CPU, as after apply_int8_quantization) may have been
    replaced or written in place, e.g. by a LoRA patch or its removal.  The new
    int8 weights and scales are written into the existing ``_w_int8`` / ``_w_scale``
    buffers, so every view of them (the stacked adaLN weights) and every cache
    keyed on their versions (the fused block's FFN weight, held as halves of one tensor) follows.
    Returns the number of layers re-quantised.
    """
    n = 0
    for _name, m in model.named_modules():
        if not (isinstance(m, nn.Linear) and getattr(m, "_int8_quantized", False) and hasattr(m, "_w_int8")):
            continue
        fp = weight_fingerprint(m.weight)
        if fp == getattr(m, "_int8_src", None):
            continue
        w_int8, w_scale = quantize_weight(m.weight.data, bool(m._int8_use_hadamard))
        m._w_int8.copy_(w_int8)
        m._w_scale.copy_(w_scale.to(m._w_scale.dtype))
        m._int8_src = fp
        n += 1
    if n:
        logger.info("INT8 refresh: %d layers re-quantised.", n)
    return n


def restore_int8_quantization(model: nn.Module) -> int:
    """Undo apply_int8_quantization (int8_linear.py:324-384); returns the module count."""
    restored = 0
    for _name, module in list(model.named_modules()):
        if not getattr(module, "_int8_quantized", False) or not isinstance(module, nn.Linear):
            continue
        target = module._w_int8.device if hasattr(module, "_w_int8") else torch.device("cpu")
        module.weight = nn.Parameter(module.weight.data.to(device=target), requires_grad=False)
        for buf in ("_w_int8", "_w_scale"):
            if buf in module._buffers:
                del module._buffers[buf]
        hook = getattr(module, "_int8_sd_hook", None)
        if hook is not None:
            hook.remove()
        for attr in ("forward", "_apply", "_int8_quantized", "_int8_use_hadamard", "_int8_layer_name",
                     "_int8_sd_hook", "_int8_src"):
            module.__dict__.pop(attr, None)
        restored += 1
    for attr in ("_int8_quantized", "_int8_stats", "_int8_lora_aware"):
        if hasattr(model, attr):
            delattr(model, attr)
    # fused block caches hold views of the removed buffers
    for m in model.modules():
        m.__dict__.pop("_zib_cache", None)
    logger.info("INT8 restore: %d modules restored.", restored)
    return restored
