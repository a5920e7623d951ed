"""CPU stand-in for the reference module ``diffusion.fp8_kernels`` — TEST INFRASTRUCTURE ONLY.

It exposes the two names the reference ``diffusion/unet.py`` imports
(unet.py:10): ``SUPPORTED_UNET_SHAPES`` and ``triton_conv2d_fp8``, computed
with the oracle (``fp8_oracle``) on the CPU instead of Triton on a GPU, so
that the reference UNet itself can run its FP8 convs on a machine without a
GPU.  Installed as ``sys.modules["diffusion.fp8_kernels"]`` before the
reference package is imported (tests/golden/make_unet_golden.py); the product
never imports it.

``triton_conv2d_fp8`` restates ``Conv2dFP8Specialized`` (fp8_kernels.py:821-913)
and the entry point (:916-923):

* forward: x and the weight are cast to bf16 (:834-836); current scaling
  quantizes both with their own amax (:858-859); delayed scaling casts with the
  given historical scales and returns the tensors' own scales (:843-853, :868-
  870); it reads the dY history max at forward time (:848) and keeps the
  history and position tensors for backward (:850-851).  Output
  ``conv(xq, wq) * sx * sw`` rounded to bf16 (:861-866).
* backward: dY in bf16 (the reference op's output dtype); current scaling
  quantizes it with its own amax; delayed casts it with the saved historical
  scale and scatters its own scale into the history at the position tensor,
  which the caller has already advanced (:883-889).  dX and dW are the
  oracle's bf16 conv gradients (:899-911).

The model here runs in fp32 (no autocast): the op's bf16 results are handed on
widened to fp32, which is the value the reference's next op sees under
autocast (group norm and the residual sum run in fp32 there too).
"""

from __future__ import annotations

import torch

import fp8_oracle as oracle

# fp8_kernels.py:17-27 (input channels, output channels, height, width)
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


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to(torch.bfloat16).contiguous()


def _quantize_delayed(t: torch.Tensor, prev: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    q, s = oracle.quantize_delayed(t, float(prev))
    return oracle.bytes_like(q, t), torch.tensor(s, dtype=torch.float32)


class _Conv2dFP8Oracle(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, hist_scales, dy_ptrs, do_delayed):
        x16, w16 = _bf16(x), _bf16(weight)
        ctx.do_delayed = do_delayed
        ctx.x_dtype, ctx.w_dtype = x.dtype, weight.dtype
        if do_delayed:
            x_scale, w_scale = (s.detach().float().reshape(()) for s in hist_scales)
            xq, x_curr = _quantize_delayed(x16, x_scale)
            wq, w_curr = _quantize_delayed(w16, w_scale)
            dy_window, window_pos = dy_ptrs
            ctx.dy_window, ctx.window_pos = dy_window, window_pos
            ctx.dy_hist = torch.max(dy_window).detach().clone()
        else:
            xq, x_scale = oracle.quantize_tensor(x16)
            wq, w_scale = oracle.quantize_tensor(w16)
        ctx.saved = (xq, wq, x_scale, w_scale)
        out = oracle.conv_fwd(xq, wq, float(x_scale), float(w_scale)).float().contiguous()
        if do_delayed:
            ctx.mark_non_differentiable(x_curr, w_curr)
            return out, x_curr, w_curr
        return out

    @staticmethod
    def backward(ctx, dy, *_):
        xq, wq, x_scale, w_scale = ctx.saved
        dy16 = _bf16(dy)
        if ctx.do_delayed:
            dy_scale = ctx.dy_hist
            dyq, dy_curr = _quantize_delayed(dy16, dy_scale)
            with torch.no_grad():
                ctx.dy_window.scatter_(0, ctx.window_pos.unsqueeze(0), dy_curr.unsqueeze(0))
        else:
            dyq, dy_scale = oracle.quantize_tensor(dy16)
        dx = oracle.conv_dx(dyq, wq, float(dy_scale), float(w_scale)).to(ctx.x_dtype).contiguous()
        dw = oracle.conv_dw(xq, dyq, float(x_scale), float(dy_scale)).to(ctx.w_dtype).contiguous()
        return dx, dw, None, None, None


def triton_conv2d_fp8(x, weight, hist_scales=None, dy_ptrs=None, do_delayed=False):
    """fp8_kernels.py:916-923 on the CPU oracle."""
    assert x.is_contiguous(memory_format=torch.channels_last)  # fp8_kernels.py:838
    if do_delayed:
        assert hist_scales is not None and dy_ptrs is not None
    return _Conv2dFP8Oracle.apply(x, weight, hist_scales, dy_ptrs, do_delayed)


__all__ = ["SUPPORTED_UNET_SHAPES", "triton_conv2d_fp8"]
