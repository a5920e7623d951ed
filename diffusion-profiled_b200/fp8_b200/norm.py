"""GroupNorm -> (FiLM) -> SiLU -> (dropout) as one differentiable op on B200.

The reference ResBlock (unet.py:149-160) computes ``silu(norm1(x))`` before
``conv_1`` and ``dropout(silu((scale + 1) * norm2(h) + shift))`` before
``conv_2`` as separate torch ops (fp32 GroupNorm under autocast, then
elementwise passes).  :func:`group_norm_act` does each chain in one statistics
pass and one apply pass over the bf16 NHWC activation (and two passes
backward), through ``fp8_b200::gn_act_fwd`` / ``gn_act_bwd``.
:class:`GroupNormActConvFP8` goes one step further where the chain feeds a
delayed-scaling FP8 conv: the apply pass writes the conv's e4m3 input directly.
"""

from __future__ import annotations

import torch
from torch.amp.autocast_mode import custom_bwd, custom_fwd

from . import ops


class GroupNormAct(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, gamma, beta, film, seed, p: float, eps: float, groups: int):
        film2 = None if film is None else film.reshape(film.shape[0], -1)
        out, stats = ops.gn_act_fwd(x, gamma, beta, film2, seed, p, eps, groups)
        ctx.save_for_backward(x, gamma, beta, film2, seed, stats)
        ctx.cfg = (p, eps, groups, None if film is None else film.shape)
        return out

    @staticmethod
    def backward(ctx, dout):
        x, gamma, beta, film2, seed, stats = ctx.saved_tensors
        p, eps, groups, film_shape = ctx.cfg
        dout = dout.to(torch.bfloat16)
        dx, dgamma, dbeta, dfilm = ops.gn_act_bwd(x, dout, gamma, beta, film2, seed, stats, p, eps, groups)
        return dx, dgamma, dbeta, _film_grad(dfilm, film_shape), None, None, None, None


def _film_grad(dfilm: torch.Tensor, film_shape):
    """The FiLM gradient in the FiLM input's shape (None without FiLM)."""
    return None if film_shape is None else dfilm.reshape(film_shape)


class GroupNormActConvFP8(torch.autograd.Function):
    """``conv3x3_fp8(dropout(silu((film_scale + 1) * GroupNorm(x) + film_shift)))`` with delayed scaling.

    The reference quantizes the conv input with the previous scale as the first
    step of its FP8 conv (Conv2dFP8Specialized.forward, fp8_kernels.py:835-845,
    on the activation of unet.py:151 / 157-159).  Here the group-norm apply pass
    writes those e4m3 bytes itself (``fp8_b200::gn_act_quant_fwd``), so the bf16
    activation is neither written nor read back; the conv and its backward are
    those of Conv2dFP8Specialized, and the activation gradient feeds the fused
    group-norm backward.  Returns ``(y, x_scale_curr, w_scale_curr)`` like the
    delayed branch of ``triton_conv2d_fp8``; the dY scale is written into
    ``dy_window`` at ``window_pos`` in backward (fp8_kernels.py:883-889)."""

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, x, gamma, beta, film, seed, weight, x_hist, w_hist, dy_window, window_pos, p: float,
                eps: float, groups: int):
        film2 = None if film is None else film.reshape(film.shape[0], -1)
        xq, x_scale_curr, stats = ops.gn_act_quant_fwd(x, gamma, beta, film2, seed, x_hist, p, eps, groups)
        w = weight.to(torch.bfloat16)
        if not w.is_contiguous(memory_format=torch.channels_last):
            w = w.contiguous(memory_format=torch.channels_last)
        wq, w_scale_curr = ops.quantize_delayed(w, w_hist)
        dy_hist = torch.max(dy_window)
        y = ops.conv3x3_fwd(xq, wq, x_hist, w_hist)
        ctx.save_for_backward(x, gamma, beta, film2, seed, stats, xq, wq, x_hist, w_hist, dy_hist)
        ctx.dy_window = dy_window
        ctx.window_pos = window_pos
        ctx.cfg = (p, eps, groups, None if film is None else film.shape)
        ctx.mark_non_differentiable(x_scale_curr, w_scale_curr)
        return y, x_scale_curr, w_scale_curr

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dy, _dx_scale, _dw_scale):
        x, gamma, beta, film2, seed, stats, xq, wq, x_hist, w_hist, dy_hist = ctx.saved_tensors
        p, eps, groups, film_shape = ctx.cfg
        dy = dy.to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
        dyq, dy_scale_curr = ops.quantize_delayed(dy, dy_hist)
        ctx.dy_window.scatter_(0, ctx.window_pos.unsqueeze(0), dy_scale_curr.unsqueeze(0))
        d_act, dw = ops.conv3x3_backward(dyq, wq, dy_hist, w_hist, xq, x_hist)  # dW beside dX
        dx, dgamma, dbeta, dfilm = ops.gn_act_bwd(x, d_act, gamma, beta, film2, seed, stats, p, eps, groups)
        return dx, dgamma, dbeta, _film_grad(dfilm, film_shape), None, dw, None, None, None, None, None, None, None


def group_norm_act(x: torch.Tensor, norm: torch.nn.GroupNorm, film: torch.Tensor | None = None,
                   p: float = 0.0, seed: torch.Tensor | None = None) -> torch.Tensor:
    """``dropout_p(silu((film_scale + 1) * norm(x) + film_shift))`` (bf16) for a bf16 or fp32 CUDA ``x``.

    ``film``: the time-embedding projection ``[N, 2C(, 1, 1)]`` (scale, shift), or None.
    ``seed``: int64 device scalar for the dropout mask (required when ``p > 0``)."""
    if p > 0.0 and seed is None:
        raise ValueError("dropout needs a seed tensor")
    x = x.contiguous(memory_format=torch.channels_last)
    return GroupNormAct.apply(x, norm.weight, norm.bias, film, seed if p > 0.0 else None, float(p),
                              float(norm.eps), int(norm.num_groups))


def fused_norm_supported(x: torch.Tensor, norm: torch.nn.GroupNorm) -> bool:
    c = x.shape[1]
    return (x.is_cuda and x.dtype in (torch.bfloat16, torch.float32) and x.dim() == 4 and c % 8 == 0 and c <= 512
            and c % norm.num_groups == 0 and norm.affine and norm.weight.dtype == torch.float32)


class LayerNormBf16(torch.autograd.Function):
    """nn.LayerNorm over the last dim with a bf16 output (``fp8_b200::layer_norm_fwd``).

    The reference's attention norm (unet.py:174, :187) runs in fp32 under autocast
    and its only consumer, the qkv projection, casts the result to bf16; this op
    returns that bf16 tensor directly and computes the parameter gradients with
    per-CTA partial sums instead of a separate column reduction."""

    @staticmethod
    def forward(ctx, x, gamma, beta, eps: float):
        y, mr = ops.layer_norm_fwd(x, gamma, beta, eps)
        ctx.save_for_backward(x, gamma, mr)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, gamma, mr = ctx.saved_tensors
        dx, dgamma, dbeta = ops.layer_norm_bwd(x, dy, gamma, mr)
        return dx, dgamma, dbeta, None


def layer_norm_bf16(x: torch.Tensor, norm: torch.nn.LayerNorm) -> torch.Tensor:
    """``norm(x)`` as bf16 for a contiguous bf16 / fp32 CUDA ``x``."""
    return LayerNormBf16.apply(x.contiguous(), norm.weight, norm.bias, float(norm.eps))


def fused_layer_norm_supported(x: torch.Tensor, norm: torch.nn.LayerNorm) -> bool:
    c = x.shape[-1]
    return (x.is_cuda and x.dtype in (torch.bfloat16, torch.float32) and c % 8 == 0 and c <= 1024
            and norm.elementwise_affine and norm.weight is not None and norm.bias is not None
            and norm.weight.dtype == torch.float32 and len(norm.normalized_shape) == 1)
