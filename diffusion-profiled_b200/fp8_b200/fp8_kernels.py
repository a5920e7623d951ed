"""Drop-in replacement for the reference module ``diffusion/fp8_kernels.py``.

Same public names, argument meanings, return values and assertion behaviour as
the reference (fattorib/diffusion-profiled, diffusion/fp8_kernels.py), backed by
the sm_100a kernels of ``libfp8ops.so`` instead of Triton.  ``unet.py`` imports
only ``SUPPORTED_UNET_SHAPES`` and ``triton_conv2d_fp8`` from here
(unet.py:10); the rest is the reference's host API, kept for callers and tests.

The Triton launch-configuration tables of the reference (DX_CONFIG_BY_SHAPE,
DW_CONFIG_BY_SHAPE) have no meaning for these kernels; DW_CONFIG_BY_SHAPE is
kept because ``conv2d_bwd_weight_fp8_prequantized(..., split_k=None)`` looks its
split count up there, and holds this build's split counts.
"""

from __future__ import annotations

from typing import Any, cast

import torch
from torch.amp.autocast_mode import custom_bwd, custom_fwd

from . import ops

FP8_DTYPE = torch.float8_e4m3fn  # fp8_kernels.py:11
FP8_MAX_E4M3 = torch.finfo(torch.float8_e4m3fn).max  # fp8_kernels.py:12 (448.0)

# (input channels, output channels, input height, input width) — fp8_kernels.py:17-27
SUPPORTED_UNET_SHAPES = (
    (128, 128, 32, 32),
    (128, 256, 32, 32),
    (256, 256, 16, 16),
    (512, 256, 16, 16),
    (256, 256, 8, 8),
    (512, 256, 8, 8),
    (512, 128, 32, 32),
    (256, 256, 32, 32),
    (256, 256, 4, 4),
)

# Split-K count of the weight-gradient kernel per shape; 0 = the library picks
# (one K split per free SM).  Same role as the reference's table at :129-139.
DW_CONFIG_BY_SHAPE: dict[tuple[int, int, int, int], int] = {shape: 0 for shape in SUPPORTED_UNET_SHAPES}


# ----------------------------------------------------------------------------- checks
def torch_checks_conv(a: torch.Tensor, b: torch.Tensor, dtype: torch.dtype) -> None:
    """fp8_kernels.py:471-476."""
    assert a.ndim == b.ndim == 4
    assert a.is_cuda and b.is_cuda and a.device == b.device
    assert a.is_contiguous() or a.is_contiguous(memory_format=torch.channels_last)
    assert b.is_contiguous() or b.is_contiguous(memory_format=torch.channels_last)


def fwd_shapes(x: torch.Tensor, weight: torch.Tensor, dtype: torch.dtype) -> tuple[int, int, int, int, int]:
    """fp8_kernels.py:479-489."""
    torch_checks_conv(x, weight, dtype)
    batch, cin, height, width = x.shape
    cout, weight_cin, kh, kw = weight.shape
    assert (weight_cin, kh, kw) == (cin, 3, 3)
    assert (cin, cout, height, width) in SUPPORTED_UNET_SHAPES, f"{(cin, cout, height, width)=}"
    return batch, cin, cout, height, width


def xgrad_shapes(dy: torch.Tensor, weight: torch.Tensor, dtype: torch.dtype) -> tuple[int, int, int, int, int]:
    """fp8_kernels.py:492-502."""
    torch_checks_conv(dy, weight, dtype)
    batch, cout, height, width = dy.shape
    weight_cout, cin, kh, kw = weight.shape
    assert (weight_cout, kh, kw) == (cout, 3, 3)
    assert (cin, cout, height, width) in SUPPORTED_UNET_SHAPES
    return batch, cin, cout, height, width


def wgrad_shapes(x: torch.Tensor, dy: torch.Tensor, dtype: torch.dtype) -> tuple[int, int, int, int, int]:
    """fp8_kernels.py:505-515."""
    torch_checks_conv(x, dy, dtype)
    batch, cin, height, width = x.shape
    dy_batch, cout, dy_height, dy_width = dy.shape
    assert (dy_batch, dy_height, dy_width) == (batch, height, width)
    assert (cin, cout, height, width) in SUPPORTED_UNET_SHAPES
    return batch, cin, cout, height, width


def torch_checks_scale(scale: torch.Tensor, device: torch.device) -> None:
    """fp8_kernels.py:667-668."""
    assert scale.device == device and scale.dtype == torch.float32 and scale.numel() == 1


# ----------------------------------------------------------------------------- quantize
def quantize_fp8_delayed(tensor: torch.Tensor, prev_scale: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Tensorwise quantization from bfloat16 to fp8 with delay (fp8_kernels.py:518-556).

    Casts with ``prev_scale`` and returns ``(fp8 tensor, scale of this tensor's amax)``.
    """
    assert tensor.dtype == torch.bfloat16 and tensor.is_cuda and tensor.ndim == 4, (
        f"{tensor.dtype} {tensor.is_cuda} {tensor.ndim}"
    )
    return ops.quantize_delayed(tensor, prev_scale)


def quantize_fp8(tensor: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Current per-tensor scaling (fp8_kernels.py:559-601): ``(fp8 tensor, amax/448)``."""
    assert tensor.dtype == torch.bfloat16 and tensor.is_cuda and tensor.ndim == 4, (
        f"{tensor.dtype} {tensor.is_cuda} {tensor.ndim}"
    )
    return ops.quantize_current(tensor)


# ----------------------------------------------------------------------------- conv forward
def conv2d_fwd_fp8_prequantized(
    x: torch.Tensor, weight: torch.Tensor, x_scale: torch.Tensor, weight_scale: torch.Tensor
) -> torch.Tensor:
    """fp8_kernels.py:604-639: bf16 channels_last ``conv(x*sx, w*sw)``, 3x3, pad 1."""
    fwd_shapes(x, weight, FP8_DTYPE)
    torch_checks_scale(x_scale, x.device)
    torch_checks_scale(weight_scale, x.device)
    return ops.conv3x3_fwd(_cl(x), _cl(weight), x_scale, weight_scale)


def _quantize_fp8_pair(x: torch.Tensor, weight: torch.Tensor):
    """quantize_fp8(x), quantize_fp8(weight) (same asserts, same bytes) in one pair of launches."""
    for t in (x, weight):
        assert t.dtype == torch.bfloat16 and t.is_cuda and t.ndim == 4, f"{t.dtype} {t.is_cuda} {t.ndim}"
    return ops.quantize_current_pair(x, weight)


def conv2d_fwd_fp8(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """fp8_kernels.py:642-650."""
    x_fp8, x_scale, weight_fp8, weight_scale = _quantize_fp8_pair(x, weight)
    return conv2d_fwd_fp8_prequantized(x_fp8, weight_fp8, x_scale, weight_scale)


def conv2d_fwd_fp8_delayed(x: torch.Tensor, weight: torch.Tensor, x_scale: torch.Tensor, w_scale: torch.Tensor):
    """fp8_kernels.py:653-664: quantize with the given (historical) scales, then conv."""
    x_fp8, _ = quantize_fp8_delayed(x, x_scale)
    weight_fp8, _ = quantize_fp8_delayed(weight, w_scale)
    return conv2d_fwd_fp8_prequantized(x_fp8, weight_fp8, x_scale, w_scale)


# ----------------------------------------------------------------------------- conv backward
def conv2d_bwd_input_fp8_prequantized(
    dy: torch.Tensor, weight: torch.Tensor, dy_scale: torch.Tensor, weight_scale: torch.Tensor
) -> torch.Tensor:
    """fp8_kernels.py:671-709: bf16 channels_last dX."""
    xgrad_shapes(dy, weight, FP8_DTYPE)
    torch_checks_scale(dy_scale, dy.device)
    torch_checks_scale(weight_scale, dy.device)
    return ops.conv3x3_dgrad(_cl(dy), _cl(weight), dy_scale, weight_scale)


def conv2d_bwd_input_fp8(dy: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """fp8_kernels.py:712-720."""
    dy_fp8, dy_scale = quantize_fp8(dy)
    weight_fp8, weight_scale = quantize_fp8(weight)
    return conv2d_bwd_input_fp8_prequantized(dy_fp8, weight_fp8, dy_scale, weight_scale)


def conv2d_bwd_weight_fp8_prequantized(
    x: torch.Tensor,
    dy: torch.Tensor,
    x_scale: torch.Tensor,
    dy_scale: torch.Tensor,
    split_k: int | None = None,
) -> torch.Tensor:
    """fp8_kernels.py:723-808: bf16 channels_last dW ``[Cout, Cin, 3, 3]``.

    Like the reference, only channels_last x and dy are implemented
    (``NotImplementedError`` otherwise, :791-792).
    """
    batch, cin, cout, height, width = wgrad_shapes(x, dy, FP8_DTYPE)
    torch_checks_scale(x_scale, x.device)
    torch_checks_scale(dy_scale, x.device)
    if split_k is None:
        split_k = DW_CONFIG_BY_SHAPE[(cin, cout, height, width)]
    if not (x.is_contiguous(memory_format=torch.channels_last) and dy.is_contiguous(memory_format=torch.channels_last)):
        raise NotImplementedError
    return ops.conv3x3_wgrad(x, dy, x_scale, dy_scale, int(split_k))


def conv2d_bwd_weight_fp8(x: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    """fp8_kernels.py:811-819."""
    x_fp8, x_scale = quantize_fp8(x)
    dy_fp8, dy_scale = quantize_fp8(dy)
    return conv2d_bwd_weight_fp8_prequantized(x_fp8, dy_fp8, x_scale, dy_scale)


def _cl(t: torch.Tensor) -> torch.Tensor:
    # The reference kernels take arbitrary strides; these kernels read NHWC
    # through TMA, so NCHW-contiguous operands are re-laid out first.
    return t if t.is_contiguous(memory_format=torch.channels_last) else t.contiguous(memory_format=torch.channels_last)


# ----------------------------------------------------------------------------- autograd op
class Conv2dFP8Specialized(torch.autograd.Function):
    """fp8_kernels.py:823-913 — FP8 3x3 conv with current or delayed scaling."""

    @staticmethod
    @custom_fwd(device_type="cuda")
    def forward(
        ctx: Any,
        x: torch.Tensor,
        weight: torch.Tensor,
        hist_scales: tuple[torch.Tensor, torch.Tensor] | None = None,
        dy_ptrs: tuple[torch.Tensor, torch.Tensor] | None = None,
        do_delayed: bool = False,
    ) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        x = x.to(torch.bfloat16)
        weight = weight.to(torch.bfloat16)

        assert x.is_contiguous(memory_format=torch.channels_last)

        ctx.do_delayed = do_delayed
        if do_delayed:
            assert hist_scales is not None
            assert dy_ptrs is not None
            x_scale, weight_scale = hist_scales
            x_fp8, x_scale_curr = quantize_fp8_delayed(x, x_scale)
            weight_fp8, weight_scale_curr = quantize_fp8_delayed(_cl(weight), weight_scale)

            dy_amax_window, window_pos = dy_ptrs
            dy_scale_hist = torch.max(dy_amax_window)

            ctx.dy_window = dy_amax_window
            ctx.window_pos = window_pos
            ctx.save_for_backward(x_fp8, weight_fp8, x_scale, weight_scale, dy_scale_hist)
        else:
            x_fp8, x_scale, weight_fp8, weight_scale = _quantize_fp8_pair(x, _cl(weight))
            ctx.save_for_backward(x_fp8, weight_fp8, x_scale, weight_scale)

        out = conv2d_fwd_fp8_prequantized(x_fp8, weight_fp8, x_scale, weight_scale)

        if do_delayed:
            ctx.mark_non_differentiable(x_scale_curr, weight_scale_curr)
            return out, x_scale_curr, weight_scale_curr
        return out

    @staticmethod
    @custom_bwd(device_type="cuda")
    def backward(ctx: Any, *grad_outputs: Any) -> Any:
        dy = cast(torch.Tensor, grad_outputs[0])
        dy = dy.contiguous(memory_format=torch.channels_last)

        if ctx.do_delayed:
            x_fp8, weight_fp8, x_scale, weight_scale, dy_scale = ctx.saved_tensors
            dy_fp8, dy_scale_curr = quantize_fp8_delayed(dy, dy_scale)
            # The window position was already advanced by the module after the
            # forward (same tensor object), so the dY scale lands one slot
            # later than the x / w scales — as in the reference (:887-889).
            window_idx = ctx.window_pos.unsqueeze(0)
            ctx.dy_window.scatter_(0, window_idx, dy_scale_curr.unsqueeze(0))
        else:
            x_fp8, weight_fp8, x_scale, weight_scale = ctx.saved_tensors
            dy_fp8, dy_scale = quantize_fp8(dy)

        assert dy_fp8.is_contiguous(memory_format=torch.channels_last)
        assert weight_fp8.is_contiguous(memory_format=torch.channels_last)
        assert x_fp8.is_contiguous(memory_format=torch.channels_last)

        # conv2d_bwd_input_fp8_prequantized and conv2d_bwd_weight_fp8_prequantized (their checks,
        # then one op that runs dW on a side stream beside dX)
        xgrad_shapes(dy_fp8, weight_fp8, FP8_DTYPE)
        batch, cin, cout, height, width = wgrad_shapes(x_fp8, dy_fp8, FP8_DTYPE)
        for scale in (dy_scale, weight_scale, x_scale):
            torch_checks_scale(scale, dy_fp8.device)
        split_k = DW_CONFIG_BY_SHAPE[(cin, cout, height, width)]
        dx, dw = ops.conv3x3_backward(dy_fp8, weight_fp8, dy_scale, weight_scale, x_fp8, x_scale, int(split_k))
        return dx, dw, None, None, None


def triton_conv2d_fp8(
    x: torch.Tensor,
    weight: torch.Tensor,
    hist_scales: tuple[torch.Tensor, torch.Tensor] | None = None,
    dy_ptrs: tuple[torch.Tensor, torch.Tensor] | None = None,
    do_delayed: bool = False,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Entry point called by ``Conv2dFP8.forward`` (unet.py:65, :74); fp8_kernels.py:916-923.

    The name is kept for drop-in compatibility; no Triton is involved.
    """
    return Conv2dFP8Specialized.apply(x, weight, hist_scales, dy_ptrs, do_delayed)


__all__ = [
    "FP8_DTYPE",
    "FP8_MAX_E4M3",
    "SUPPORTED_UNET_SHAPES",
    "DW_CONFIG_BY_SHAPE",
    "torch_checks_conv",
    "fwd_shapes",
    "xgrad_shapes",
    "wgrad_shapes",
    "torch_checks_scale",
    "quantize_fp8_delayed",
    "quantize_fp8",
    "conv2d_fwd_fp8_prequantized",
    "conv2d_fwd_fp8",
    "conv2d_fwd_fp8_delayed",
    "conv2d_bwd_input_fp8_prequantized",
    "conv2d_bwd_input_fp8",
    "conv2d_bwd_weight_fp8_prequantized",
    "conv2d_bwd_weight_fp8",
    "Conv2dFP8Specialized",
    "triton_conv2d_fp8",
]
