"""FP8 self-attention for the UNet's attention blocks (``attn_fwd_fp8_kernel`` / ``attn_bwd_kernel``).

Stands in for ``F.scaled_dot_product_attention(q, k, v)`` of ``CHWAttention``
(diffusion/unet.py:189-199), where q, k, v are the three thirds of the qkv
projection's output split into heads of 64 channels.  The op takes that output
as it is, ``qkv [B, L, 3C]``, and returns ``o [B, L, C]`` with head h in columns
``h*64 .. h*64+63`` -- the tensor the output projection reads -- so no head
transposes are made on either side.

Forward: q, k, v quantized to e4m3 per (image, head) (amax/448 scales), QK^T
and PV on the FP8 tensor cores, fp32 softmax, P as e4m3(p * 448).  Backward:
the gradient with straight-through quantizers on the bf16 tensor cores.  The
sequence length must be a multiple of 16 up to 256 and the head size 64 (the
UNet's 16x16 and 4x4 attention: L = 256 and 16, 4 heads of 64).
"""

from __future__ import annotations

import torch

from . import _lib
from .ops import _ptr, _require_cuda, _stream

HEAD_DIM = 64
MAX_SEQ = 256


def attention_supported(qkv: torch.Tensor, heads: int) -> bool:
    """Whether ``fp8_attention`` takes this qkv projection output."""
    if qkv.dim() != 3 or not qkv.is_cuda or qkv.dtype != torch.bfloat16:
        return False
    b, seq, c3 = qkv.shape
    return (c3 == 3 * heads * HEAD_DIM and 16 <= seq <= MAX_SEQ and seq % 16 == 0
            and qkv.stride(2) == 1 and qkv.stride(1) % 8 == 0 and qkv.stride(0) == seq * qkv.stride(1)
            and qkv.data_ptr() % 16 == 0)


def _check(qkv: torch.Tensor, heads: int) -> tuple[int, int, int]:
    if not attention_supported(qkv, heads):
        raise RuntimeError(f"fp8 attention: unsupported qkv {tuple(qkv.shape)} {qkv.dtype} "
                           f"strides {qkv.stride()} for {heads} heads of {HEAD_DIM}")
    b, seq, _ = qkv.shape
    return b, seq, qkv.stride(1)


@torch.library.custom_op("fp8_b200::attention_fwd", mutates_args=())
def attention_fwd(qkv: torch.Tensor, heads: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """-> (o [B, L, C] bf16, lse [B, heads, L] fp32, scales [B, heads, 4] fp32)."""
    dev = _require_cuda(qkv)
    b, seq, ld = _check(qkv, heads)
    c = heads * HEAD_DIM
    o = torch.empty(b, seq, c, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(b, heads, seq, device=dev, dtype=torch.float32)
    scales = torch.empty(b, heads, 4, device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().fp8_attention_fwd(_ptr(qkv), _ptr(o), _ptr(lse), _ptr(scales), b, seq, heads,
                                                 HEAD_DIM, ld, c, _stream(dev)), "fp8_attention_fwd")
    return o, lse, scales


@attention_fwd.register_fake
def _(qkv, heads):
    b, seq, _ = qkv.shape
    return (qkv.new_empty(b, seq, heads * HEAD_DIM), qkv.new_empty(b, heads, seq, dtype=torch.float32),
            qkv.new_empty(b, heads, 4, dtype=torch.float32))


@torch.library.custom_op("fp8_b200::attention_bwd", mutates_args=())
def attention_bwd(qkv: torch.Tensor, o: torch.Tensor, do: torch.Tensor, lse: torch.Tensor, scales: torch.Tensor,
                  heads: int) -> torch.Tensor:
    """-> d(qkv), bf16 in qkv's shape."""
    dev = _require_cuda(qkv, o, do, lse, scales)
    b, seq, ld = _check(qkv, heads)
    c = heads * HEAD_DIM
    for t, shape in ((o, (b, seq, c)), (do, (b, seq, c))):
        if t.dtype != torch.bfloat16 or tuple(t.shape) != shape or not t.is_contiguous():
            raise RuntimeError(f"fp8 attention backward: expected contiguous bf16 {shape}, got {tuple(t.shape)}")
    dqkv = torch.empty(b, seq, 3 * c, device=dev, dtype=torch.bfloat16)
    if ld != 3 * c:
        raise RuntimeError("fp8 attention backward: qkv rows must be dense")
    with torch.cuda.device(dev):
        _lib.check(_lib.load().fp8_attention_bwd(_ptr(qkv), _ptr(o), _ptr(do), _ptr(lse.contiguous()),
                                                 _ptr(scales.contiguous()), _ptr(dqkv), b, seq, heads, HEAD_DIM,
                                                 ld, c, _stream(dev)), "fp8_attention_bwd")
    return dqkv


@attention_bwd.register_fake
def _(qkv, o, do, lse, scales, heads):
    return torch.empty_like(qkv, memory_format=torch.contiguous_format)


class FP8Attention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv: torch.Tensor, heads: int) -> torch.Tensor:
        o, lse, scales = attention_fwd(qkv, heads)
        ctx.save_for_backward(qkv, o, lse, scales)
        ctx.heads = heads
        return o

    @staticmethod
    def backward(ctx, do: torch.Tensor):
        qkv, o, lse, scales = ctx.saved_tensors
        return attention_bwd(qkv, o, do.to(torch.bfloat16).contiguous(), lse, scales, ctx.heads), None


def fp8_attention(qkv: torch.Tensor, heads: int) -> torch.Tensor:
    """``o [B, L, C]`` = multi-head softmax(q k^T / 8) v of the qkv projection output ``[B, L, 3C]``."""
    return FP8Attention.apply(qkv, heads)


__all__ = ["attention_supported", "attention_fwd", "attention_bwd", "FP8Attention", "fp8_attention"]
