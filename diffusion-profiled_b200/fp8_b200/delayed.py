"""Delayed-scaling FP8 convs with the scale histories kept and updated on the device.

The reference keeps, per FP8 conv, three scale histories (``amax_window_acts``,
``amax_window_weights``, ``amax_window_dy``, 1024 scales each) and a position
(unet.py:50-56, 69-91; fp8_kernels.py:841-853, 883-889).  Every call it takes
``torch.max`` of each history, casts with those scales, scatters the new x / w
scales at the position, advances it, and in backward scatters the dY scale at
the advanced position -- eight small launches per conv besides the casts.  Here
the cast kernels take the max of the history themselves and the one-CTA
finalize that computes a tensor's scale writes it into the history and steps
the position (``fp8_b200::quantize_delayed_window`` / ``gn_act_quant_fwd_window``),
so the histories, the scales used and the bytes are the same and the
bookkeeping costs no launch of its own.
"""

from __future__ import annotations

import torch
from torch.amp.autocast_mode import custom_bwd, custom_fwd

from . import ops


def _weight_bf16(weight: torch.Tensor) -> torch.Tensor:
    w = weight.to(torch.bfloat16)
    return w if w.is_contiguous(memory_format=torch.channels_last) else w.contiguous(memory_format=torch.channels_last)


def hand_off_dy(conv, db: torch.Tensor, dbq: torch.Tensor, sdy: torch.Tensor) -> None:
    """Give the FP8 conv module ``conv`` the e4m3 cast of its output gradient ``db``, made (with the
    history update) by the op that produced ``db``; its backward then skips its own quantize."""
    conv._dy_handoff = (db, dbq, sdy)


def hand_off_skip_grad(conv, x: torch.Tensor, dx: torch.Tensor) -> None:
    """Give the fused group-norm conv ``conv`` (whose normalised input is ``x``) a second gradient of x,
    which its backward adds to the norm's input gradient (``gn_act_bwd(..., dx_add=dx)``); the producer
    of ``dx`` then returns no gradient for x itself."""
    conv._dx_add = (x.data_ptr(), x.shape, x.dtype, dx)


def _take_dx_add(owner, x: torch.Tensor):
    entry = getattr(owner, "_dx_add", None) if owner is not None else None
    if entry is None:
        return None
    owner._dx_add = None
    ptr, shape, dtype, dx = entry
    if ptr != x.data_ptr() or shape != x.shape or dtype != x.dtype:
        # the producer returned no gradient for x, so dropping this one would lose it
        raise RuntimeError("the skip gradient handed to this conv belongs to another tensor")
    return dx


def _take_dy(owner, dy: torch.Tensor):
    """(dyq, sdy) handed to ``owner`` for exactly this gradient tensor, else None.  The entry holds
    ``db`` alive, so equal storage, shape and strides mean it is that tensor."""
    entry = getattr(owner, "_dy_handoff", None) if owner is not None else None
    if entry is None:
        return None
    owner._dy_handoff = None
    db, dbq, sdy = entry
    if (dy.data_ptr() == db.data_ptr() and dy.dtype == db.dtype and dy.shape == db.shape
            and dy.stride() == db.stride()):
        return dbq, sdy
    return None


def _conv_backward(ctx, dy, xq, wq, sx, sw):
    pre = _take_dy(ctx.owner, dy)
    if pre is not None:  # cast (and its history update) done by the producer of dy
        dyq, sdy = pre
    else:
        dy = dy.to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
        # the dY scale lands at the position the forward already advanced (fp8_kernels.py:883-889)
        dyq, sdy = ops.quantize_delayed_window(dy, ctx.win_dy, ctx.pos, False)
    # an fp32 weight gets the bf16 dW widened by the reduce pass, not by an autograd cast
    widen = ctx.w_dtype == torch.float32
    # weights re-laid out for the data-grad by the step's batched transpose, when it made them;
    # dW runs on a side stream beside dX
    return ops.conv3x3_backward(dyq, wq, sdy, sw, xq, sx, 0, widen, ctx.wq_t)


def _weight_q(ctx, weight, win_w, pos, pre):
    """The e4m3 weight and its scale: from the step's batched weight quantize when given
    (``pre = (wq, sw, wq_t)``, history written, position to be stepped here; wq_t the data-grad
    layout or None), else quantized now.  Sets ``ctx.wq_t``."""
    if pre is not None:
        ctx.wq_t = pre[2]
        return pre[0], pre[1]
    ctx.wq_t = None
    return ops.quantize_delayed_window(_weight_bf16(weight), win_w, pos, False)


class ConvFP8Delayed(torch.autograd.Function):
    """``Conv2dFP8Specialized`` (delayed branch) plus the module's history update, on device histories."""

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, x, weight, win_x, win_w, win_dy, pos, pre=None, owner=None):
        ctx.owner = owner
        x = x.to(torch.bfloat16)
        wq, sw = _weight_q(ctx, weight, win_w, pos, pre)
        xq, sx = ops.quantize_delayed_window(x, win_x, pos, True)
        ctx.save_for_backward(xq, wq, sx, sw)
        ctx.win_dy, ctx.pos, ctx.w_dtype = win_dy, pos, weight.dtype
        return ops.conv3x3_fwd(xq, wq, sx, sw)

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dy):
        xq, wq, sx, sw = ctx.saved_tensors
        dx, dw = _conv_backward(ctx, dy, xq, wq, sx, sw)
        return dx, dw, None, None, None, None, None, None


class GroupNormActConvFP8Delayed(torch.autograd.Function):
    """``GroupNormActConvFP8`` on device histories: the group-norm pass casts with max(win_x)."""

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx, x, gamma, beta, film, seed, weight, win_x, win_w, win_dy, pos, p: float, eps: float,
                groups: int, pre=None, owner=None, x_owner=None):
        ctx.owner = owner
        # x_owner: the delayed FP8 conv whose (bf16) output x is; the norm's backward then also makes
        # the e4m3 cast of x's gradient for that conv's backward
        ctx.x_owner = x_owner if x.dtype == torch.bfloat16 else None
        film2 = None if film is None else film.reshape(film.shape[0], -1)
        wq, sw = _weight_q(ctx, weight, win_w, pos, pre)
        xq, sx, stats = ops.gn_act_quant_fwd_window(x, gamma, beta, film2, seed, win_x, pos, True, p, eps, groups)
        ctx.save_for_backward(x, gamma, beta, film2, seed, stats, xq, wq, sx, sw)
        ctx.win_dy, ctx.pos, ctx.w_dtype = win_dy, pos, weight.dtype
        ctx.cfg = (p, eps, groups, None if film is None else film.shape)
        return ops.conv3x3_fwd(xq, wq, sx, sw)

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx, dy):
        x, gamma, beta, film2, seed, stats, xq, wq, sx, sw = ctx.saved_tensors
        p, eps, groups, film_shape = ctx.cfg
        d_act, dw = _conv_backward(ctx, dy, xq, wq, sx, sw)
        conv = ctx.x_owner
        dx_add = _take_dx_add(ctx.owner, x)  # the identity skip's gradient of x, from the residual join
        if dx_add is not None:
            dx, dgamma, dbeta, dfilm = ops.gn_act_bwd(x, d_act, gamma, beta, film2, seed, stats, p, eps, groups,
                                                      dx_add)
        elif conv is not None:
            dx, dgamma, dbeta, dfilm, dxq, sdx = ops.gn_act_bwd_quant(
                x, d_act, gamma, beta, film2, seed, stats, p, eps, groups, conv.amax_window_dy, conv.window_pos)
            hand_off_dy(conv, dx, dxq, sdx)
        else:
            dx, dgamma, dbeta, dfilm = ops.gn_act_bwd(x, d_act, gamma, beta, film2, seed, stats, p, eps, groups)
        dfilm = None if film_shape is None else dfilm.reshape(film_shape)
        return dx, dgamma, dbeta, dfilm, None, dw, None, None, None, None, None, None, None, None, None, None


def quantize_conv_weights(convs) -> None:
    """Quantize the weights of delayed-scaling FP8 conv modules in one batch (three launches).

    Each module then finds ``(wq, sw)`` in ``_pre_weight`` for its next forward.  The weight
    histories are written at the modules' positions, which the modules' activation quantize
    then uses and steps, exactly as a per-call weight quantize would leave them."""
    if not convs:
        return
    weights = []
    for m in convs:
        w = m.conv.weight.detach()
        weights.append(w if w.is_contiguous(memory_format=torch.channels_last)
                       else w.contiguous(memory_format=torch.channels_last))
    out = ops.quantize_weights_delayed(weights, [m.amax_window_weights for m in convs],
                                       [m.window_pos for m in convs])
    k = len(convs)
    # the data-grad layout of the weights whose data-grad does not read them in place, one launch
    relayout = [i for i, m in enumerate(convs) if getattr(m, "dgrad_relayout", False)]
    wq_t = dict(zip(relayout, ops.transpose_conv_weights([out[i] for i in relayout])))
    for i, m in enumerate(convs):
        m._pre_weight = (out[i], out[k + i], wq_t.get(i))


__all__ = ["ConvFP8Delayed", "GroupNormActConvFP8Delayed", "quantize_conv_weights", "hand_off_dy",
           "hand_off_skip_grad"]
