"""Nearest-neighbour resampling and skip concatenation of the UNet as single passes.

The reference UNet (unet.py:366-383) downsamples with
``F.interpolate(x, scale_factor=0.5, mode="nearest")``, upsamples with
``scale_factor=2.0`` and concatenates the skip with ``torch.cat(dim=1)``.  Under
bf16 autocast ``F.interpolate`` runs in fp32 (its input is cast up first, its
output is fp32) and ``torch.cat`` promotes to the wider dtype, so those lines
cost a cast pass, a resampling pass and a concatenation copy.
:func:`downsample_nearest` and :func:`upsample_cat` produce the same values and
dtypes in one read and one write per element (``fp8_b200::resample_down2`` /
``up_cat`` and their backward ops).  :func:`residual_join` does the residual
``(skip + h) / math.sqrt(2.0)`` the same way.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import ops
from .delayed import hand_off_dy, hand_off_skip_grad

_FLOATS = (torch.bfloat16, torch.float32)


class _Down2(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        ctx.shape = (x.shape[2], x.shape[3], x.dtype == torch.float32)
        return ops.resample_down2(x)

    @staticmethod
    def backward(ctx, dy):
        h, w, x_fp32 = ctx.shape
        return ops.resample_down2_bwd(dy, h, w, x_fp32)


class _UpCat(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, s, factor: int, out_fp32: bool):
        ctx.cfg = (a.shape[1], factor, a.dtype == torch.float32, s.dtype == torch.float32)
        return ops.up_cat(a, s, factor, out_fp32)

    @staticmethod
    def backward(ctx, dy):
        c1, factor, a_fp32, s_fp32 = ctx.cfg
        da, ds = ops.up_cat_bwd(dy, c1, factor, a_fp32, s_fp32)
        return da, ds, None, None


class _UpCatPair(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, s, factor: int):
        ctx.cfg = (a.shape[1], factor, a.dtype == torch.float32, s.dtype == torch.float32)
        return ops.up_cat_pair(a, s, factor)

    @staticmethod
    def backward(ctx, dy, dy16):
        c1, factor, a_fp32, s_fp32 = ctx.cfg
        da, ds = ops.up_cat_pair_bwd(dy, dy16, c1, factor, a_fp32, s_fp32)
        return da, ds, None


def resample_supported(*ts: torch.Tensor) -> bool:
    return all(t.is_cuda and t.dim() == 4 and t.dtype in (torch.bfloat16, torch.float32) and t.shape[1] % 8 == 0
               and t.is_contiguous(memory_format=torch.channels_last) for t in ts)


def downsample_nearest(x: torch.Tensor) -> torch.Tensor:
    """``F.interpolate(x, scale_factor=0.5, mode="nearest")`` as bf16 autocast computes it (fp32 out)."""
    if not (resample_supported(x) and x.shape[2] % 2 == 0 and x.shape[3] % 2 == 0
            and (torch.is_autocast_enabled("cuda") or x.dtype == torch.float32)):
        return torch.nn.functional.interpolate(x, scale_factor=0.5, mode="nearest")
    return _Down2.apply(x)


def upsample_cat(a: torch.Tensor, s: torch.Tensor, factor: int) -> torch.Tensor:
    """``torch.cat([F.interpolate(a, scale_factor=factor, mode="nearest") if factor > 1 else a, s], dim=1)``."""
    autocast = torch.is_autocast_enabled("cuda")
    if not resample_supported(a, s) or factor not in (1, 2):
        up = torch.nn.functional.interpolate(a, scale_factor=float(factor), mode="nearest") if factor > 1 else a
        return torch.cat([up, s], dim=1)
    up_fp32 = a.dtype == torch.float32 or (factor > 1 and autocast)
    return _UpCat.apply(a, s, factor, up_fp32 or s.dtype == torch.float32)


def upsample_cat_pair(a: torch.Tensor, s: torch.Tensor, factor: int) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``(y, y.to(torch.bfloat16))`` for ``y = upsample_cat(a, s, factor)`` when y is fp32 (bf16
    autocast), both from one pass; ``(y, None)`` otherwise.  The bf16 copy is what autocast gives
    the 1x1 skip conv of the block that reads y (unet.py:139, 161)."""
    autocast = torch.is_autocast_enabled("cuda")
    if resample_supported(a, s) and factor in (1, 2) and autocast:
        if a.dtype == torch.float32 or s.dtype == torch.float32 or factor > 1:
            return _UpCatPair.apply(a, s, factor)
    return upsample_cat(a, s, factor), None


class _AddScale(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a, b, inv: float, dy_target=None, skip_target=None):
        ctx.cfg = (a.dtype, b.dtype, inv)
        ctx.dy_target = dy_target
        ctx.skip_target = skip_target
        if skip_target is not None:
            ctx.save_for_backward(a)
        return ops.add_scale(a, b, inv)

    @staticmethod
    def backward(ctx, dy):
        ta, tb, inv = ctx.cfg
        conv = ctx.dy_target
        if conv is not None and tb == torch.bfloat16 and dy.dim() == 4:
            da, db, dbq, sdy = ops.add_scale_bwd_quant(dy, inv, ta == torch.float32, conv.amax_window_dy,
                                                       conv.window_pos)
            hand_off_dy(conv, db, dbq, sdy)
        else:
            da, db = ops.add_scale_bwd(dy, inv, ta == torch.float32, tb == torch.float32)
        if ctx.skip_target is not None:  # a's gradient is added by the norm's backward of the block's conv_1
            (a,) = ctx.saved_tensors
            hand_off_skip_grad(ctx.skip_target, a, da)
            da = None
        return da, db, None, None, None


def _same_dense_layout(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.shape != b.shape or a.stride() != b.stride():
        return False
    return a.is_contiguous() or (a.dim() == 4 and a.is_contiguous(memory_format=torch.channels_last))


def residual_join(a: torch.Tensor, b: torch.Tensor, divisor: float = math.sqrt(2.0), dy_target=None,
                  skip_target=None) -> torch.Tensor:
    """``(a + b) / divisor`` as one pass, with the dtype and the two roundings of the torch ops (unet.py:161, :203).

    ``dy_target``: the delayed-scaling FP8 conv module whose output is ``b``; the backward then also
    writes the e4m3 cast of b's gradient, with that conv's dY history update, and hands it over
    (fp8_b200.delayed.hand_off_dy).  ``skip_target``: the fused group-norm conv whose normalised input is
    ``a`` itself; a's gradient is then added inside that conv's norm backward instead of by autograd
    (fp8_b200.delayed.hand_off_skip_grad)."""
    if not (a.is_cuda and b.is_cuda and a.dtype in _FLOATS and b.dtype in _FLOATS and _same_dense_layout(a, b)
            and a.numel() % 8 == 0 and a.numel() > 0):
        return (a + b) / divisor
    inv = float(np.float32(1.0) / np.float32(divisor))  # torch: a host scalar divisor becomes an fp32 reciprocal
    return _AddScale.apply(a, b, inv, dy_target, skip_target)


__all__ = ["downsample_nearest", "upsample_cat", "upsample_cat_pair", "resample_supported", "residual_join"]
