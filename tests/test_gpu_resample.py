"""GPU parity: the UNet's nearest resampling + skip concatenation kernels
(fp8_b200.resample) against F.interpolate / torch.cat under bf16 autocast, as the
reference calls them (unet.py:366-383).

Resampling copies values, so the forward outputs (values and dtypes) must be
identical; the downsample gradient too.  The upsample gradient sums 2x2 blocks
in fp32, where the summation order may differ from torch's: within one rounding
step of the gradient's dtype."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _t(shape, dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to(dtype).to(device).contiguous(memory_format=torch.channels_last)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(128, 256, 32, 32), (4, 128, 16, 16), (3, 8, 2, 6)])
def test_downsample_matches_interpolate_under_autocast(cuda, shape, dtype):
    from fp8_b200.resample import downsample_nearest

    x0 = _t(shape, dtype, sum(shape), cuda)
    dy = _t((shape[0], shape[1], shape[2] // 2, shape[3] // 2), torch.float32, 7, cuda)
    outs = []
    for fn in (downsample_nearest, lambda x: F.interpolate(x, scale_factor=0.5, mode="nearest")):
        x = x0.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = fn(x)
        y.backward(dy)
        outs.append((y.detach(), x.grad))
    (y1, g1), (y2, g2) = outs
    assert y1.dtype == y2.dtype == torch.float32 and torch.equal(y1, y2)
    assert g1.dtype == g2.dtype == dtype and torch.equal(g1, g2)


@pytest.mark.parametrize("factor", [1, 2])
@pytest.mark.parametrize("da,ds", [(torch.float32, torch.bfloat16), (torch.bfloat16, torch.bfloat16),
                                   (torch.float32, torch.float32), (torch.bfloat16, torch.float32)])
def test_upsample_cat_matches_torch_under_autocast(cuda, factor, da, ds):
    from fp8_b200.resample import upsample_cat

    n, c1, c2, h = 8, 256, 128, 32
    a0 = _t((n, c1, h // factor, h // factor), da, 11, cuda)
    s0 = _t((n, c2, h, h), ds, 12, cuda)
    outs = []
    for fused in (True, False):
        a = a0.clone().requires_grad_(True)
        s = s0.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            if fused:
                y = upsample_cat(a, s, factor)
            else:
                up = F.interpolate(a, scale_factor=2.0, mode="nearest") if factor > 1 else a
                y = torch.cat([up, s], dim=1)
        dy = _t(y.shape, y.dtype, 13, cuda)
        y.backward(dy)
        outs.append((y.detach(), a.grad, s.grad))
    (y1, a1, s1), (y2, a2, s2) = outs
    assert y1.dtype == y2.dtype and torch.equal(y1, y2)
    assert s1.dtype == s2.dtype == ds and torch.equal(s1, s2)
    assert a1.dtype == a2.dtype == da
    tol = 2.0 ** -7 if da == torch.bfloat16 else 1e-6
    assert ((a1.float() - a2.float()).abs() <= tol * a2.float().abs() + 1e-30).all()


@pytest.mark.parametrize("factor", [1, 2])
@pytest.mark.parametrize("da,ds", [(torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32),
                                   (torch.float32, torch.float32)])
def test_upsample_cat_pair_matches_cat_and_autocast_copy(cuda, factor, da, ds):
    """upsample_cat_pair = (cat of the upsampled a and s, its bf16 copy) bit for bit, and its backward takes
    the sum of both outputs' gradients as autograd forms it: ds bitwise, da within one rounding step."""
    from fp8_b200.resample import upsample_cat_pair

    if factor == 1 and da == ds == torch.bfloat16:
        pytest.skip("no fp32 output: the pair is not formed")
    n, c1, c2, h = 8, 256, 128, 16
    a0 = _t((n, c1, h // factor, h // factor), da, 21, cuda)
    s0 = _t((n, c2, h, h), ds, 22, cuda)
    dy = _t((n, c1 + c2, h, h), torch.float32, 23, cuda)
    dy16 = _t((n, c1 + c2, h, h), torch.bfloat16, 24, cuda)
    outs = []
    for fused in (True, False):
        a = a0.clone().requires_grad_(True)
        s = s0.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            if fused:
                y, y16 = upsample_cat_pair(a, s, factor)
            else:
                up = F.interpolate(a, scale_factor=2.0, mode="nearest") if factor > 1 else a
                y = torch.cat([up, s], dim=1)
                y16 = y.to(torch.bfloat16)
        torch.autograd.backward([y, y16], [dy, dy16])
        outs.append((y.detach(), y16.detach(), a.grad, s.grad))
    (y1, q1, a1, s1), (y2, q2, a2, s2) = outs
    assert y1.dtype == y2.dtype == torch.float32 and torch.equal(y1, y2)
    assert q1.dtype == q2.dtype == torch.bfloat16 and torch.equal(q1, q2)
    assert q1.is_contiguous(memory_format=torch.channels_last)
    assert s1.dtype == s2.dtype == ds and torch.equal(s1, s2)
    assert a1.dtype == a2.dtype == da
    tol = 2.0 ** -7 if da == torch.bfloat16 else 1e-6
    assert ((a1.float() - a2.float()).abs() <= tol * a2.float().abs() + 1e-30).all()


def test_unet_with_paired_skip_cast_matches_separate_cast(cuda):
    """The UNet with the up stages' skip-conv copy made by the up_cat pass: the same output bytes, and
    gradients within bf16 rounding of the separate cast + gradient sum."""
    from fp8_b200.train import build_model

    x = (torch.rand(4, 3, 32, 32) * 2 - 1).to(cuda).contiguous(memory_format=torch.channels_last)
    t = torch.randint(0, 1000, (4,)).to(cuda)
    res = []
    for paired in (True, False):
        m = build_model(fp8=False, device=cuda, seed=0, p_drop=0.0)
        m.config.fused_skip_cast = paired
        with torch.no_grad():  # the zero-initialised branches would give zero gradients everywhere
            torch.manual_seed(1)
            for mod in m.modules():
                if isinstance(mod, torch.nn.Conv2d) and not mod.weight.any():
                    torch.nn.init.normal_(mod.weight, std=0.02)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = m(x, t)
        y.float().square().mean().backward()
        res.append((y.detach(), m.conv_in.weight.grad.clone(), m.up_stages[-1].blocks[0].skip_connection.weight.grad))
    (ya, ia, sa), (yb, ib, sb) = res
    assert torch.equal(ya, yb)
    for u, v in ((ia, ib), (sa, sb)):
        assert ((u - v).abs().max() / v.abs().max()).item() <= 1e-2


def test_unet_forward_identical_with_fused_resampling(cuda):
    """The whole UNet forward gives the same bytes with the fused resampling (it only copies values)."""
    from fp8_b200.train import build_model

    x = (torch.rand(4, 3, 32, 32) * 2 - 1).to(cuda).contiguous(memory_format=torch.channels_last)
    t = torch.randint(0, 1000, (4,)).to(cuda)
    ys = []
    for fused in (True, False):
        m = build_model(fp8=False, device=cuda, seed=0, fused_resample=fused).eval()
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
            ys.append(m(x, t))
    assert torch.equal(ys[0], ys[1])


@pytest.mark.parametrize("ta,tb", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.bfloat16),
                                   (torch.bfloat16, torch.float32), (torch.float32, torch.float32)])
def test_residual_join_matches_torch_bitwise(cuda, ta, tb):
    """(a + b) / math.sqrt(2.0) as the reference's ops compute it, forward and backward, bit for bit."""
    import math

    from fp8_b200.resample import residual_join

    a0 = _t((16, 256, 16, 16), ta, 21, cuda)
    b0 = _t((16, 256, 16, 16), tb, 22, cuda)
    res = []
    for fused in (True, False):
        a = a0.clone().requires_grad_(True)
        b = b0.clone().requires_grad_(True)
        y = residual_join(a, b) if fused else (a + b) / math.sqrt(2.0)
        dy = _t(y.shape, y.dtype, 23, cuda)
        y.backward(dy)
        res.append((y.detach(), a.grad, b.grad))
    for u, v in zip(*res):
        assert u.dtype == v.dtype and torch.equal(u, v)


@pytest.mark.parametrize("ta,ty", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32)])
def test_join_backward_quantize_matches_separate_quantize(cuda, ta, ty):
    """add_scale_bwd_quant = add_scale_bwd + the FP8 conv's backward quantize of db
    (quantize_delayed_window(db, window, pos, advance=False)): same gradients, e4m3 bytes, scale used,
    history and position."""
    from fp8_b200 import ops

    dy = _t((8, 256, 16, 16), ty, 31, cuda)
    inv = 0.70710677
    res = []
    for fused in (True, False):
        win = torch.zeros(16, device=cuda)
        win[:5] = torch.tensor([1e-3, 4e-3, 2e-3, 0.0, 1e-4])
        pos = torch.tensor(3, dtype=torch.int64, device=cuda)
        if fused:
            da, db, dbq, used = ops.add_scale_bwd_quant(dy, inv, ta == torch.float32, win, pos)
        else:
            da, db = ops.add_scale_bwd(dy, inv, ta == torch.float32, False)
            dbq, used = ops.quantize_delayed_window(db, win, pos, False)
        res.append((da, db, dbq.view(torch.uint8), used, win, pos))
    for u, v in zip(*res):
        assert u.dtype == v.dtype and torch.equal(u, v)
    assert res[0][0].dtype == ta and res[0][1].dtype == torch.bfloat16
    assert res[0][5].item() == 3  # the position is not stepped


def test_dy_handoff_is_taken_once_and_only_for_its_tensor(cuda):
    from fp8_b200.delayed import _take_dy, hand_off_dy
    from fp8_b200.unet import Conv2dFP8

    conv = Conv2dFP8(128, 128, True, "delayed", 16).to(cuda)
    db = torch.randn(2, 128, 8, 8, device=cuda).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    dbq = torch.zeros_like(db, dtype=torch.float8_e4m3fn)
    s = torch.tensor(0.5, device=cuda)
    hand_off_dy(conv, db, dbq, s)
    assert _take_dy(conv, db.clone()) is None  # another tensor: not used, and the entry is dropped
    assert _take_dy(conv, db) is None
    hand_off_dy(conv, db, dbq, s)
    got = _take_dy(conv, db)
    assert got is not None and got[0] is dbq and got[1] is s
    assert _take_dy(conv, db) is None  # taken once
