"""GPU parity: fused GroupNorm -> FiLM -> SiLU -> dropout (fp8_b200.norm) against
the same chain in fp32 torch ops on the same bf16 inputs.

Tolerance: max|got - ref| / max|ref| <= 1e-2 (bf16 outputs of fp32 arithmetic)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

TOL = 1e-2
SHAPES = [(128, 32, 32), (256, 16, 16), (384, 32, 32), (512, 8, 8), (512, 4, 4), (256, 32, 32), (128, 8, 8)]


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def _inputs(n, c, h, w, film: bool, seed: int, device, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(n, c, h, w, generator=g) * 2 + 0.5).to(dtype)
    x = x.contiguous(memory_format=torch.channels_last).to(device)
    norm = torch.nn.GroupNorm(32, c).to(device)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.2 * torch.randn(c, generator=g))
        norm.bias.copy_(0.1 * torch.randn(c, generator=g))
    f = (0.3 * torch.randn(n, 2 * c, 1, 1, generator=g)).to(torch.bfloat16).to(device) if film else None
    dout = torch.randn(n, c, h, w, generator=g).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    return x, norm, f, dout.to(device)


def _reference(x, norm, film, mask=None, p=0.0):
    z = F.group_norm(x.float(), norm.num_groups, norm.weight, norm.bias, norm.eps)
    if film is not None:
        s, t = torch.chunk(film.float(), 2, dim=1)
        z = (s + 1) * z + t
    a = F.silu(z)
    if mask is not None:
        a = a * mask / (1 - p)
    return a


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("film", [False, True])
@pytest.mark.parametrize("c,h,w", SHAPES)
def test_group_norm_act_forward_and_backward(cuda, c, h, w, film, dtype):
    """bf16 input (after a conv) and fp32 input (after autocast's fp32 resampling)."""
    from fp8_b200.norm import group_norm_act

    x, norm, f, dout = _inputs(4, c, h, w, film, seed=c + h + film, device=cuda, dtype=dtype)
    xr = x.detach().clone().requires_grad_(True)
    fr = None if f is None else f.detach().clone().requires_grad_(True)
    x.requires_grad_(True)
    if f is not None:
        f.requires_grad_(True)
    out = group_norm_act(x, norm, f)
    assert out.dtype == torch.bfloat16 and out.is_contiguous(memory_format=torch.channels_last)
    ref_norm = torch.nn.GroupNorm(32, c).to(cuda)
    ref_norm.load_state_dict(norm.state_dict())
    ref = _reference(xr, ref_norm, fr)
    assert _rel(out, ref) <= TOL
    out.backward(dout)
    ref.backward(dout.float())
    assert x.grad.dtype == dtype
    assert _rel(x.grad, xr.grad) <= TOL
    assert _rel(norm.weight.grad, ref_norm.weight.grad) <= TOL
    assert _rel(norm.bias.grad, ref_norm.bias.grad) <= TOL
    if f is not None:
        assert f.grad.shape == f.shape and _rel(f.grad, fr.grad) <= TOL


def test_group_norm_act_dropout(cuda):
    from fp8_b200.norm import group_norm_act

    p = 0.1
    x, norm, f, dout = _inputs(8, 256, 16, 16, True, seed=5, device=cuda)
    seed = torch.tensor(1234, dtype=torch.int64, device=cuda)
    x.requires_grad_(True)
    out = group_norm_act(x, norm, f, p=p, seed=seed)
    again = group_norm_act(x.detach(), norm, f, p=p, seed=seed)
    assert torch.equal(out, again)  # the mask is a function of (seed, element)
    other = group_norm_act(x.detach(), norm, f, p=p, seed=seed + 1)
    assert not torch.equal(out, other)
    ref_nodrop = _reference(x.detach(), norm, f)
    mask = ((out != 0) | (ref_nodrop == 0)).float()
    dropped = 1.0 - mask.mean().item()
    assert abs(dropped - p) < 0.01, dropped
    xr = x.detach().clone().requires_grad_(True)
    ref = _reference(xr, norm, f, mask=mask, p=p)
    assert _rel(out, ref) <= TOL
    out.backward(dout)
    ref.backward(dout.float())
    assert _rel(x.grad, xr.grad) <= TOL


def test_group_norm_act_large_offset_statistics(cuda):
    """Channels with a large common offset: the shifted sums keep the variance accurate."""
    from fp8_b200.norm import group_norm_act

    x, norm, _, _ = _inputs(2, 128, 32, 32, False, seed=9, device=cuda)
    x = (x.float() * 0.05 + 40.0).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    out = group_norm_act(x, norm)
    assert _rel(out, _reference(x, norm, None)) <= TOL
