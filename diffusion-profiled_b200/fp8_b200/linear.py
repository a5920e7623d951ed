"""Scaled FP8 linear — the "scaled FP8 GEMM" of the hot path.

The reference has no FP8 linear kernel: its attention qkv/out projections
(unet.py:171-172), ``TimeEmbed.mlp`` (unet.py:101) and the time-embedding MLP
(unet.py:331-336) are bf16 ``nn.Linear(bias=False)`` layers under autocast, and
the author lists FP8 linears as future work (extra/post.md:230).  This op gives
them the same per-tensor e4m3 treatment as the reference convs:

    forward   y  = (Xq @ Wq^T) * sx * sw (+ b)               quantize X, W (current scaling)
    backward  dX = (dYq @ Wq)   * sdy * sw                   quantize dY
              dW = (dYq^T @ Xq) * sdy * sx
              db = sum_m dY                                  (bf16, only with a bias)

``weight`` has the ``nn.Linear`` layout ``[out_features, in_features]``.
"""

from __future__ import annotations

from typing import Any

import torch
from torch.amp.autocast_mode import custom_bwd, custom_fwd

from . import ops


class _FP8LinearFn(torch.autograd.Function):
    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(ctx: Any, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, silu: bool):
        x2 = x.to(torch.bfloat16).reshape(-1, x.shape[-1]).contiguous()
        w = weight.to(torch.bfloat16).contiguous()
        xq, sx, wq, sw = ops.quantize_current_pair(x2, w)
        b = None if bias is None else bias.to(torch.bfloat16).contiguous()
        if silu and b is None:
            raise RuntimeError("the fused SiLU epilogue needs a bias")
        epi = ops.EPILOGUE_NONE if b is None else (ops.EPILOGUE_BIAS_SILU if silu else ops.EPILOGUE_BIAS)
        y = ops.gemm(xq, wq, sx, sw, b, epi)
        ctx.save_for_backward(xq, wq, sx, sw, b)
        ctx.has_bias = bias is not None
        ctx.silu = silu
        ctx.x_shape = x.shape
        return y.reshape(*x.shape[:-1], weight.shape[0])

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx: Any, dy: torch.Tensor):
        xq, wq, sx, sw, b = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1]).to(torch.bfloat16)
        if ctx.silu:
            # y = silu(z): the pre-activation z is recomputed by one more GEMM
            # instead of being kept alive from the forward.
            z = ops.gemm(xq, wq, sx, sw, b, ops.EPILOGUE_BIAS).float()
            sig = torch.sigmoid(z)
            dy2 = (dy2.float() * sig * (1 + z * (1 - sig))).to(torch.bfloat16)
        dy2 = dy2.contiguous()
        dyq, sdy = ops.quantize_current(dy2)
        wt = ops.transpose_2d(wq)  # [in, out]
        dx = ops.gemm(dyq, wt, sdy, sw).reshape(ctx.x_shape)
        dw = ops.gemm_wgrad(dyq, xq, sdy, sx)
        db = dy2.float().sum(0).to(torch.bfloat16) if ctx.has_bias else None
        return dx, dw, db, None


def fp8_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None = None,
    *,
    scaling: str = "current",
    silu: bool = False,
) -> torch.Tensor:
    """``y = x @ weight.T (+ bias)`` with e4m3 operands and fp32 accumulation, bf16 output.

    ``scaling`` must be ``"current"`` (per-call amax of X, W and dY).
    ``silu=True`` fuses ``silu(y)`` into the GEMM epilogue (requires a bias).
    """
    if scaling != "current":
        raise ValueError(f"unsupported FP8 linear scaling {scaling!r} (only 'current')")
    return _FP8LinearFn.apply(x, weight, bias, silu)


class FP8Linear(torch.nn.Linear):
    """``nn.Linear`` whose matmul runs through :func:`fp8_linear` (same parameters / state_dict)."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:  # noqa: D102
        return fp8_linear(x, self.weight, self.bias)

    @classmethod
    def from_linear(cls, lin: torch.nn.Linear) -> "FP8Linear":
        new = cls.__new__(cls)
        torch.nn.Module.__init__(new)
        new.in_features, new.out_features = lin.in_features, lin.out_features
        new.weight = lin.weight
        new.bias = lin.bias
        return new


def swap_linears(module: torch.nn.Module, predicate=None) -> int:
    """Replace ``nn.Linear`` children (recursively) by :class:`FP8Linear` sharing their parameters.

    Only layers whose shapes the GEMM supports (in % 128 == 0, out % 128 == 0) are
    swapped; returns the number swapped.
    """
    count = 0
    for name, child in list(module.named_children()):
        if isinstance(child, torch.nn.Linear) and not isinstance(child, FP8Linear):
            ok = child.in_features % 128 == 0 and child.out_features % 128 == 0
            if ok and (predicate is None or predicate(name, child)):
                setattr(module, name, FP8Linear.from_linear(child))
                count += 1
        else:
            count += swap_linears(child, predicate)
    return count


__all__ = ["fp8_linear", "FP8Linear", "swap_linears"]
