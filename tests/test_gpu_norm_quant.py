"""GPU parity: group norm -> (FiLM) -> SiLU -> (dropout) fused with the delayed
e4m3 quantize of its output, and the residual-block conv built on it.

Bars: the e4m3 bytes and the current scale equal, bit for bit, the CPU oracle's
delayed quantize (fp8_oracle.quantize_delayed, the restatement of
quantize_fp8_delayed, fp8_kernels.py:518-556) of the bf16 activation that the
unfused group-norm op writes; the fused residual-block conv gives the same
forward bytes, input and norm gradients as the unfused path, and dW within one
bf16 rounding step (its split-K additions have no fixed order)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fp8_oracle as oracle

pytestmark = pytest.mark.gpu

SHAPES = [(128, 32, 32), (256, 16, 16), (256, 32, 32), (512, 8, 8), (512, 16, 16)]


def _inputs(n, c, h, w, film, seed, device, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(n, c, h, w, generator=g) * 2 + 0.5).to(dtype).contiguous(memory_format=torch.channels_last)
    norm = torch.nn.GroupNorm(32, c)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.2 * torch.randn(c, generator=g))
        norm.bias.copy_(0.1 * torch.randn(c, generator=g))
    f = (0.3 * torch.randn(n, 2 * c, generator=g)).to(torch.bfloat16) if film else None
    return x.to(device), norm.to(device), None if f is None else f.to(device)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("film,p", [(False, 0.0), (True, 0.0), (True, 0.1)])
@pytest.mark.parametrize("c,h,w", SHAPES)
def test_gn_act_quant_matches_oracle_on_the_unfused_activation(cuda, c, h, w, film, p, dtype):
    from fp8_b200 import ops

    x, norm, f = _inputs(4, c, h, w, film, seed=c + h + int(10 * p), device=cuda, dtype=dtype)
    seed = torch.tensor(1234 + c, dtype=torch.int64, device=cuda) if p > 0 else None
    args = (x, norm.weight, norm.bias, f, seed)
    a, stats_ref = ops.gn_act_fwd(*args, p, norm.eps, 32)
    amax = a.float().abs().max().item()
    for prev in (amax / 448.0 * 0.7, amax / 448.0 * 3.0, 0.0, 2.0 ** -70):
        prev_t = torch.tensor(prev, dtype=torch.float32, device=cuda)
        q, s_curr, stats = ops.gn_act_quant_fwd(*args, prev_t, p, norm.eps, 32)
        q_ref, s_ref = oracle.quantize_delayed(a.cpu(), np.float32(prev))
        got = q.cpu().view(torch.uint8).permute(0, 2, 3, 1).reshape(-1).numpy()
        assert np.array_equal(got, q_ref), f"prev={prev}: {np.count_nonzero(got != q_ref)} bytes differ"
        assert s_curr.item() == float(s_ref)
        assert torch.equal(stats, stats_ref)
    assert ops.device_error() == 0


def _block_pair(cuda, cin, cout, fused):
    from fp8_b200.unet import ResidualBlock, UNetConfig

    cfg = UNetConfig(fp8_convs_enabled=True, fp8_scaling_type="delayed", fused_norm=True, p_drop=0.1)
    torch.manual_seed(0)
    blk = ResidualBlock(cfg, cin, cout, p_drop=0.1).to(cuda).to(memory_format=torch.channels_last)
    with torch.no_grad():
        torch.nn.init.normal_(blk.conv_2.conv.weight, std=0.02)
        for m in (blk.conv_1, blk.conv_2):  # calibrated windows, as after warm-up
            m.amax_window_acts.fill_(0.01)
            m.amax_window_weights.fill_(0.0005)
            m.amax_window_dy.fill_(1e-5)
        blk.dropout_seed.fill_(77)
    if not fused:  # the unfused path: group norm op, then the FP8 conv module with the torch bookkeeping
        from fp8_b200.norm import group_norm_act

        for m in (blk.conv_1, blk.conv_2):
            m.device_scale_history = False
            m.forward_normed = (lambda mod: lambda x, norm, film=None, p=0.0, seed=None, x_owner=None:
                                mod(group_norm_act(x, norm, film, p, seed)))(m)
    return blk


@pytest.mark.parametrize("cin,cout,h", [(128, 128, 32), (128, 256, 16), (256, 256, 16)])
def test_fused_residual_block_matches_unfused(cuda, cin, cout, h):
    """ResidualBlock with delayed scaling, three steps: the group-norm pass writing the e4m3 input and
    the device-side scale histories (GroupNormActConvFP8Delayed) vs group_norm_act + Conv2dFP8 with
    the reference's torch.max / scatter bookkeeping.  Same output bytes, histories and positions."""
    g = torch.Generator().manual_seed(cin + h)
    x0 = torch.randn(4, cin, h, h, generator=g).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    t0 = torch.randn(4, 512, generator=g).to(torch.bfloat16)
    dout = (torch.randn(4, cout, h, h, generator=g) * 0.1).to(torch.bfloat16).contiguous(
        memory_format=torch.channels_last)
    res = {}
    for fused in (True, False):
        blk = _block_pair(cuda, cin, cout, fused)
        for it in range(3):  # the histories advance and their maxima change between steps
            x = (x0 * (1.0 + 0.5 * it)).to(cuda).requires_grad_(True)
            t = t0.to(cuda)
            blk.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                y = blk(x, t)
            y.backward(dout.to(cuda) * (1.0 + it))
        torch.cuda.synchronize()
        res[fused] = dict(
            y=y.detach(), dx=x.grad.detach(),
            g1=blk.norm1.weight.grad, b1=blk.norm1.bias.grad, g2=blk.norm2.weight.grad, b2=blk.norm2.bias.grad,
            temb=blk.t_embed_wb.mlp.weight.grad, w1=blk.conv_1.conv.weight.grad, w2=blk.conv_2.conv.weight.grad,
            win=torch.cat([m.amax_window_acts[:5] for m in (blk.conv_1, blk.conv_2)]
                          + [m.amax_window_dy[:5] for m in (blk.conv_1, blk.conv_2)]
                          + [m.amax_window_weights[:5] for m in (blk.conv_1, blk.conv_2)]
                          + [m.window_pos.view(1).float() for m in (blk.conv_1, blk.conv_2)]),
        )
    a, b = res[True], res[False]
    assert torch.equal(a["y"], b["y"])
    assert torch.equal(a["win"], b["win"])
    # dW of conv_2 feeds nothing else; conv_1's input gradient goes through conv_2's dX only
    for k in ("w1", "w2"):
        ref = b[k].float()
        excess = (a[k].float() - ref).abs() - (2.0 ** -7 * ref.abs() + 1e-4 * ref.abs().max())
        assert excess.max().item() <= 0.0, k
    for k in ("dx", "g1", "b1", "g2", "b2", "temb"):
        assert oracle.max_rel_err(a[k], b[k]) <= 1e-6, k


def test_device_scale_history_matches_torch_bookkeeping(cuda):
    """Conv2dFP8 (delayed) alone: ConvFP8Delayed vs the reference's bookkeeping around triton_conv2d_fp8,
    over several steps (the dY scale lands one slot after the x / w scales, as in the reference)."""
    from fp8_b200.unet import Conv2dFP8

    g = torch.Generator().manual_seed(5)
    x0 = torch.randn(8, 256, 16, 16, generator=g).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    mods = []
    for dev_hist in (True, False):
        torch.manual_seed(0)
        m = Conv2dFP8(256, 256, True, "delayed", 1024, device_scale_history=dev_hist).to(cuda)
        with torch.no_grad():
            m.window_pos.fill_(1022)  # wraps around during the test
        mods.append(m)
    outs = {}
    for m, key in zip(mods, ("device", "torch")):
        ys = []
        for it in range(4):
            x = (x0 * (1.0 + it)).to(cuda).requires_grad_(True)
            y = m(x)
            y.backward(torch.ones_like(y) * 1e-3 * (it + 1))
            ys.append((y.detach(), x.grad))
        torch.cuda.synchronize()
        outs[key] = (ys, m.amax_window_acts.clone(), m.amax_window_weights.clone(), m.amax_window_dy.clone(),
                     m.window_pos.clone())
    a, b = outs["device"], outs["torch"]
    for (ya, ga), (yb, gb) in zip(a[0], b[0]):
        assert torch.equal(ya, yb) and torch.equal(ga, gb)
    for u, v in zip(a[1:], b[1:]):
        assert torch.equal(u, v)


def test_batched_weight_quantize_matches_per_conv(cuda):
    """UNet forward/backward steps with the per-step batched weight quantize give the same outputs,
    histories and positions as quantizing each weight inside its conv (the first forward of a model)."""
    from fp8_b200.train import build_model
    from fp8_b200.unet import Conv2dFP8

    x = (torch.rand(4, 3, 32, 32) * 2 - 1).to(cuda).contiguous(memory_format=torch.channels_last)
    t = torch.randint(0, 1000, (4,)).to(cuda)
    runs = []
    for batched in (True, False):
        m = build_model(fp8=True, scaling="delayed", device=cuda, seed=0, p_drop=0.0)
        outs = []
        for step in range(3):
            if not batched:
                m._fp8_delayed_convs = None  # every step quantizes inside the convs
            with torch.autocast("cuda", dtype=torch.bfloat16):
                y = m(x * (1 + step), t)
            y.float().square().mean().backward()
            outs.append(y.detach())
        convs = [c for c in m.modules() if isinstance(c, Conv2dFP8)]
        hist = torch.cat([torch.cat([c.amax_window_weights[:4], c.amax_window_acts[:4], c.amax_window_dy[:4],
                                     c.window_pos.view(1).float()]) for c in convs])
        grads = torch.cat([c.conv.weight.grad.flatten()[:64].float() for c in convs if c.conv.weight.grad is not None])
        runs.append((outs, hist, grads))
    (oa, ha, ga), (ob, hb, gb) = runs
    for u, v in zip(oa, ob):
        assert torch.equal(u, v)
    assert torch.equal(ha, hb)
    assert ((ga - gb).abs() <= 2.0 ** -7 * gb.abs() + 1e-4 * gb.abs().max()).all()


@pytest.mark.parametrize("film,p", [(False, 0.0), (True, 0.1)])
@pytest.mark.parametrize("c,h,w", [(128, 32, 32), (256, 16, 16), (256, 8, 8)])
def test_gn_act_bwd_quant_matches_bwd_then_conv_quantize(cuda, c, h, w, film, p):
    """gn_act_bwd_quant = gn_act_bwd + the backward quantize of the FP8 conv that produced x
    (quantize_delayed_window(dx, window, pos, advance=False)): the same gradients, e4m3 bytes, scale
    used, history and position."""
    from fp8_b200 import ops

    x, norm, f = _inputs(4, c, h, w, film, seed=c + h + 3, device=cuda)
    seed = torch.tensor(99, dtype=torch.int64, device=cuda) if p > 0 else None
    _, stats = ops.gn_act_fwd(x, norm.weight, norm.bias, f, seed, p, norm.eps, 32)
    g = torch.Generator().manual_seed(c)
    dy = (torch.randn(x.shape, generator=g) * 1e-2).to(torch.bfloat16).to(cuda).contiguous(
        memory_format=torch.channels_last)
    res = []
    for fused in (True, False):
        win = torch.zeros(32, device=cuda)
        win[:3] = torch.tensor([2e-6, 1e-5, 5e-6])
        pos = torch.tensor(7, dtype=torch.int64, device=cuda)
        args = (x, dy, norm.weight, norm.bias, f, seed, stats, p, norm.eps, 32)
        if fused:
            dx, dg, db, dfilm, dxq, used = ops.gn_act_bwd_quant(*args, win, pos)
        else:
            dx, dg, db, dfilm = ops.gn_act_bwd(*args)
            dxq, used = ops.quantize_delayed_window(dx, win, pos, False)
        res.append((dx, dg, db, dfilm, dxq.view(torch.uint8), used, win, pos))
    for u, v in zip(*res):
        assert u.dtype == v.dtype and torch.equal(u, v)
    assert res[0][7].item() == 7
    assert ops.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gn_act_bwd_with_skip_gradient_matches_autograd_sum(cuda, dtype):
    """gn_act_bwd(..., dx_add) = gn_act_bwd(...) + dx_add as autograd sums the two gradients of a tensor
    read twice (in x's dtype), bit for bit."""
    from fp8_b200 import ops

    x, norm, f = _inputs(4, 256, 16, 16, True, seed=11, device=cuda, dtype=dtype)
    seed = torch.tensor(5, dtype=torch.int64, device=cuda)
    _, stats = ops.gn_act_fwd(x, norm.weight, norm.bias, f, seed, 0.1, norm.eps, 32)
    g = torch.Generator().manual_seed(12)
    dy = (torch.randn(x.shape, generator=g) * 1e-2).to(torch.bfloat16).to(cuda).contiguous(
        memory_format=torch.channels_last)
    add = (torch.randn(x.shape, generator=g) * 1e-2).to(dtype).to(cuda).contiguous(memory_format=torch.channels_last)
    args = (x, dy, norm.weight, norm.bias, f, seed, stats, 0.1, norm.eps, 32)
    dx, dg, db, dfilm = ops.gn_act_bwd(*args)
    dx2, dg2, db2, dfilm2 = ops.gn_act_bwd(*args, add)
    assert torch.equal(dx2, dx + add)
    assert torch.equal(dg2, dg) and torch.equal(db2, db) and torch.equal(dfilm2, dfilm)
