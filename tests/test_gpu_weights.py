"""GPU parity: the batched fp32 <-> bf16 weight casts (fp8_b200.weights) equal torch's casts bit for bit,
and the UNet with them computes what it computes with autocast's per-weight casts."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_cast_batch_matches_torch_casts(cuda):
    from fp8_b200 import ops

    g = torch.Generator().manual_seed(3)
    sizes = [1, 3, 8, 4097, 8192, 8192 * 3 + 5, 300_001]
    src = [(torch.randn(n, generator=g) * 10.0 ** (i - 3)).to(cuda) for i, n in enumerate(sizes)]
    src.append(torch.randn(4101, generator=g).to(cuda)[1:])  # 4 bytes off 16-byte alignment: scalar loop
    src.append(torch.tensor([0.0, -0.0, 1e-40, 3.4e38, float("inf"), -float("inf"), 1.0 + 2.0 ** -8,
                             1.0 + 3 * 2.0 ** -8], device=cuda))  # subnormal, overflow to inf, ties
    out = ops.cast_batch(src, True)
    for s, o in zip(src, out):
        assert o.dtype == torch.bfloat16 and torch.equal(o.view(torch.int16), s.to(torch.bfloat16).view(torch.int16))
    back = ops.cast_batch(out, False)
    for o, b in zip(out, back):
        assert b.dtype == torch.float32 and torch.equal(b, o.float())
    many = [torch.randn(100 + i, generator=g).to(cuda) for i in range(70)]  # more than one call's 64
    for s, o in zip(many, ops.cast_batch(many, True)):
        assert torch.equal(o, s.to(torch.bfloat16))


def test_cast_batch_keeps_channels_last_strides(cuda):
    from fp8_b200 import ops

    w = torch.randn(256, 512, 3, 3, device=cuda).contiguous(memory_format=torch.channels_last)
    (o,) = ops.cast_batch([w], True)
    assert o.stride() == w.stride() and torch.equal(o, w.to(torch.bfloat16))


def test_cast_cat_matches_cat_then_cast(cuda):
    from fp8_b200 import ops
    from fp8_b200.weights import cast_cat_weights_bf16

    g = torch.Generator().manual_seed(4)
    ws = [torch.randn(r, 512, generator=g).to(cuda).requires_grad_(True) for r in (256, 512, 1024, 256)]
    y = cast_cat_weights_bf16(ws)
    assert torch.equal(y, torch.cat([w.detach() for w in ws]).to(torch.bfloat16))
    gy = torch.randn_like(y)
    y.backward(gy)
    r0 = 0
    for w in ws:
        assert torch.equal(w.grad, gy[r0:r0 + w.shape[0]].float())
        r0 += w.shape[0]
    assert ops.cast_cat_bf16([w.detach() for w in ws]).shape == (2048, 512)


def test_unet_with_batched_weight_casts_matches_autocast_casts(cuda):
    """One batched cast of the bf16 layers' weights (and of their gradients back): the same UNet output bytes,
    and weight gradients within the run-to-run spread of the bf16 kernels."""
    from fp8_b200.train import build_model
    from fp8_b200.unet import CHWAttention

    x = (torch.rand(4, 3, 32, 32) * 2 - 1).to(cuda).contiguous(memory_format=torch.channels_last)
    t = torch.randint(0, 1000, (4,)).to(cuda)
    res = []
    for batched in (True, False):
        m = build_model(fp8=False, device=cuda, seed=0, p_drop=0.0)
        m.config.batched_weight_cast = batched
        with torch.no_grad():  # the zero-initialised branches would give zero gradients everywhere
            torch.manual_seed(1)
            for mod in m.modules():
                if isinstance(mod, (torch.nn.Conv2d, torch.nn.Linear)) and not mod.weight.any():
                    torch.nn.init.normal_(mod.weight, std=0.02)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = m(x, t)
        y.float().square().mean().backward()
        attn = [a for a in m.modules() if isinstance(a, CHWAttention)][0]
        grads = [attn.qkv.weight.grad, attn.out.weight.grad, m.time_embed[0].weight.grad,
                 m.up_stages[-1].blocks[0].skip_connection.weight.grad,
                 m.down_stages[0].blocks[0].t_embed_wb.mlp.weight.grad]
        assert all(gr is not None and gr.dtype == torch.float32 for gr in grads)
        res.append((y.detach(), [gr.clone() for gr in grads]))
    (ya, ga), (yb, gb) = res
    assert torch.equal(ya, yb)
    for u, v in zip(ga, gb):
        assert ((u - v).abs().max() / v.abs().max()).item() <= 1e-2
