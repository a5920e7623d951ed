"""GPU parity: the attention-block LayerNorm (fp8_b200.norm.layer_norm_bf16)
against torch's fp32 nn.LayerNorm on the same inputs (the reference runs it in
fp32 under autocast, unet.py:187, and the qkv projection casts it to bf16).

Tolerances: y within one bf16 rounding of the fp32 result (max relative error
over the tensor <= 2^-8); dx, dgamma, dbeta max|got - ref| / max|ref| <= 1e-2."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("tokens,c", [(32768, 256), (8192, 512), (1000, 200), (777, 1024), (16, 8), (3, 128)])
def test_layer_norm_forward_backward(cuda, tokens, c, dtype):
    from fp8_b200.norm import layer_norm_bf16

    g = torch.Generator().manual_seed(tokens + c)
    x0 = (torch.randn(tokens, c, generator=g) * 1.5 + 0.3).to(dtype)
    ln = torch.nn.LayerNorm(c)
    with torch.no_grad():
        ln.weight.copy_(1 + 0.3 * torch.randn(c, generator=g))
        ln.bias.copy_(0.2 * torch.randn(c, generator=g))
    ln = ln.to(cuda)
    dy = torch.randn(tokens, c, generator=g).to(torch.bfloat16).to(cuda)

    x = x0.to(cuda).requires_grad_(True)
    y = layer_norm_bf16(x, ln)
    assert y.dtype == torch.bfloat16 and y.shape == x.shape
    y.backward(dy)
    dgamma, dbeta = ln.weight.grad.clone(), ln.bias.grad.clone()
    ln.weight.grad = None
    ln.bias.grad = None

    xr = x0.to(cuda).float().requires_grad_(True)
    yr = F.layer_norm(xr, (c,), ln.weight, ln.bias, ln.eps)
    yr.backward(dy.float())
    assert _rel(y, yr) <= 2.0 ** -8
    assert x.grad.dtype == dtype and _rel(x.grad, xr.grad) <= 1e-2
    assert _rel(dgamma, ln.weight.grad) <= 1e-2
    assert _rel(dbeta, ln.bias.grad) <= 1e-2


def test_layer_norm_parameter_gradients_are_deterministic(cuda):
    from fp8_b200 import ops

    g = torch.Generator().manual_seed(3)
    x = torch.randn(32768, 256, generator=g).to(torch.bfloat16).to(cuda)
    dy = torch.randn(32768, 256, generator=g).to(torch.bfloat16).to(cuda)
    gamma = torch.ones(256, device=cuda)
    beta = torch.zeros(256, device=cuda)
    _, mr = ops.layer_norm_fwd(x, gamma, beta, 1e-5)
    a = ops.layer_norm_bwd(x, dy, gamma, mr)
    b = ops.layer_norm_bwd(x, dy, gamma, mr)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_attention_block_uses_the_fused_norm(cuda):
    """CHWAttention with the fused norm vs the reference's fp32 nn.LayerNorm path, under autocast."""
    from fp8_b200.unet import CHWAttention, UNetConfig

    torch.manual_seed(0)
    blk = CHWAttention(UNetConfig(fused_norm=True), 256).to(cuda)
    torch.nn.init.normal_(blk.out.weight, std=0.02)
    ref = CHWAttention(UNetConfig(fused_norm=False), 256).to(cuda)
    ref.load_state_dict(blk.state_dict())
    x0 = torch.randn(8, 256, 16, 16, device=cuda).contiguous(memory_format=torch.channels_last)
    outs = []
    for m in (blk, ref):
        x = x0.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = m(x)
        y.float().square().mean().backward()
        outs.append((y.detach(), x.grad, m.norm.weight.grad, m.qkv.weight.grad))
    for a, b in zip(*outs):
        assert _rel(a, b) <= 2e-2
