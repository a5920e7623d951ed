"""bf16 copies of the UNet's bf16-layer weights, made in one launch per step.

Under bf16 autocast every fp32 weight that a bf16 layer reads is cast by its own
launch (torch's autocast cast cache holds one copy per weight and step), and in
backward every bf16 weight gradient is cast back to fp32 by another.  For the
reference UNet these are the attention qkv / out projections (unet.py:171-172),
the 1x1 skip convs (:139), the blocks' time-embedding projections (:101) and the
time-embedding MLP (:331-336): about 40 small launches per step each way.
:func:`cast_weights_bf16` and :func:`cast_cat_weights_bf16` make the same bf16
values in one launch (``fp8_b200::cast_batch`` / ``cast_cat_bf16``) and their
backward casts the gradients back in one launch; the layers then receive bf16
weights, on which autocast makes no copy.
"""

from __future__ import annotations

import torch

from . import ops


def _dense(t: torch.Tensor) -> torch.Tensor:
    return t if ops._dense(t) else t.contiguous()


class _CastEach(torch.autograd.Function):
    @staticmethod
    def forward(ctx, *weights):
        ctx.set_materialize_grads(False)
        return tuple(ops.cast_batch(list(weights), True))

    @staticmethod
    def backward(ctx, *grads):
        idx = [i for i, g in enumerate(grads) if g is not None]
        out = [None] * len(grads)
        for i, g in zip(idx, ops.cast_batch([_dense(grads[i]) for i in idx], False)):
            out[i] = g
        return tuple(out)


class _CastCat(torch.autograd.Function):
    @staticmethod
    def forward(ctx, *weights):
        ctx.rows = [w.shape[0] for w in weights]
        return ops.cast_cat_bf16(list(weights))

    @staticmethod
    def backward(ctx, g):
        g = g.contiguous()
        return tuple(ops.cast_batch(list(torch.split(g, ctx.rows, dim=0)), False))


def cast_weights_bf16(weights: list[torch.Tensor]) -> list[torch.Tensor]:
    """``[w.to(torch.bfloat16) for w in weights]`` (dense fp32 CUDA tensors), differentiable, one launch
    each way."""
    if not weights:
        return []
    return list(_CastEach.apply(*[_dense(w) for w in weights]))


def cast_cat_weights_bf16(weights: list[torch.Tensor]) -> torch.Tensor:
    """``torch.cat(weights, dim=0).to(torch.bfloat16)`` for contiguous 2-D fp32 weights of one width."""
    return _CastCat.apply(*weights)


def batch_cast_applies(weights: list[torch.Tensor]) -> bool:
    """Whether the layers reading these weights run in bf16 autocast on CUDA with fp32 weights."""
    return (bool(weights) and torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16
            and all(w.is_cuda and w.dtype == torch.float32 for w in weights))


__all__ = ["cast_weights_bf16", "cast_cat_weights_bf16", "batch_cast_applies"]
