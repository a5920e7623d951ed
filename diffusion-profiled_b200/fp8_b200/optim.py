"""Gradient clipping + AdamW + the EMA of the weights as one pass (``fp8_adamw_ema_step``).

The reference training step ends with ``clip_grad_norm_(params, 1.0)``, a fused
AdamW step and the EMA update of ddpm.py:20-25 -- three passes over 32 M
parameters plus a norm reduction.  :class:`FusedAdamWEMA` does them in three
kernels that read and write each parameter, gradient, moment and EMA value once;
the step count lives on the device so a captured CUDA graph advances it on every
replay.  Same formulas as ``torch.optim.AdamW`` (decoupled weight decay, bias
corrections, ``exp_avg.lerp_``); fp32 rounding may differ in the last bits.
"""

from __future__ import annotations

from ctypes import c_int64, c_void_p

import torch

from . import _lib


class FusedAdamWEMA:
    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 1e-2,
                 max_grad_norm: float | None = None, ema: list[torch.Tensor] | None = None, ema_beta: float = 0.9999):
        self.params = [p for p in params if p.requires_grad]
        if not self.params:
            raise ValueError("no trainable parameters")
        for p in self.params:
            if p.dtype != torch.float32 or not p.is_cuda or not _dense(p):
                raise ValueError("FusedAdamWEMA needs dense fp32 CUDA parameters")
        if ema is not None and (len(ema) != len(self.params) or any(
                e.shape != p.shape or e.stride() != p.stride() or e.dtype != torch.float32
                for e, p in zip(ema, self.params))):
            raise ValueError("one fp32 EMA tensor per parameter, with the parameter's shape and layout")
        self.ema = ema
        self.lr, self.betas, self.eps, self.weight_decay = float(lr), betas, float(eps), float(weight_decay)
        self.max_grad_norm = float(max_grad_norm) if max_grad_norm else 0.0
        self.ema_beta = float(ema_beta)
        dev = self.params[0].device
        self.exp_avg = [torch.zeros_like(p) for p in self.params]
        self.exp_avg_sq = [torch.zeros_like(p) for p in self.params]
        self.step_count = torch.zeros((), device=dev, dtype=torch.float32)
        count = len(self.params)
        self._n = (c_int64 * count)(*[p.numel() for p in self.params])
        lib = _lib.load()
        self._ws = torch.empty((max(lib.fp8_adamw_ema_workspace_bytes(count, self._n) // 4, 4),), device=dev,
                               dtype=torch.float32)

    def zero_grad(self, set_to_none: bool = True) -> None:
        for p in self.params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    @torch.no_grad()
    def step(self) -> None:
        grads = []
        for p in self.params:
            g = p.grad
            if g is None:
                raise RuntimeError("every parameter needs a gradient before the fused step")
            if g.dtype != torch.float32 or g.stride() != p.stride():
                g = _like(p, g)
                p.grad = g
            grads.append(g)
        count = len(self.params)
        arr = lambda ts: (c_void_p * count)(*[0 if t is None else t.data_ptr() for t in ts])  # noqa: E731
        ema = arr(self.ema) if self.ema is not None else None
        b1, b2 = self.betas
        dev = self.params[0].device
        with torch.cuda.device(dev):
            _lib.call("fp8_adamw_ema_step", count, arr(self.params), arr(grads), arr(self.exp_avg),
                      arr(self.exp_avg_sq), ema, self._n, c_void_p(self.step_count.data_ptr()), self.lr, b1, b2,
                      self.eps, self.weight_decay, self.ema_beta, self.max_grad_norm,
                      c_void_p(self._ws.data_ptr()), self._ws.numel() * 4,
                      c_void_p(torch.cuda.current_stream(dev).cuda_stream))


def _dense(t: torch.Tensor) -> bool:
    return t.is_contiguous() or (t.dim() == 4 and t.is_contiguous(memory_format=torch.channels_last))


def _like(p: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    """g as fp32 with p's memory layout (the kernel walks all tensors of a parameter in one order)."""
    out = torch.empty_like(p)
    out.copy_(g)
    return out


__all__ = ["FusedAdamWEMA"]
