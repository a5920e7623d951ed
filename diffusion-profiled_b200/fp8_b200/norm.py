"""GroupNorm -> (FiLM) -> SiLU -> (dropout) as one differentiable op on B200.

The reference ResBlock (unet.py:149-160) computes ``silu(norm1(x))`` before
``conv_1`` and ``dropout(silu((scale + 1) * norm2(h) + shift))`` before
``conv_2`` as separate torch ops (fp32 GroupNorm under autocast, then
elementwise passes).  :func:`group_norm_act` does each chain in one statistics
pass and one apply pass over the bf16 NHWC activation (and two passes
backward), through ``fp8_b200::gn_act_fwd`` / ``gn_act_bwd``.
"""

from __future__ import annotations

import torch

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
        dx, totals = ops.gn_act_bwd(x, dout, gamma, beta, film2, seed, stats, p, eps, groups)
        c = x.shape[1]
        sc = 1.0 if film2 is None else film2[:, :c].float() + 1.0
        t_df, t_dfz, t_dfx = totals.unbind(1)  # [N, C] each
        dgamma = (sc * t_dfx).sum(0)
        dbeta = (sc * t_df).sum(0)
        dfilm = None
        if film2 is not None:
            dfilm = torch.cat([t_dfz, t_df], dim=1).to(film2.dtype).reshape(film_shape)
        return dx, dgamma, dbeta, dfilm, None, None, None, None


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
