"""GPU parity of the FP8 attention kernels against the oracle.

``fp8_attention`` replaces ``F.scaled_dot_product_attention`` of the attention
blocks (diffusion/unet.py:189-199; 16x16: L = 256, 4x4 middle stage: L = 16,
4 heads of 64).  The oracle (oracle/fp8_oracle.py ``attention_fwd`` /
``attention_bwd``) restates what the kernels compute: per (image, head) e4m3
quantize of q, k, v with amax/448 scales, fp32 softmax, P as e4m3(p * 448),
and the straight-through backward with P and dS rounded to bf16.

Bars: scales bit-exact; o, dq, dk, dv within max relative error 1e-2 (the
contract's fp32-accumulation tolerance; exp and summation order differ between
the kernel and the CPU); lse within 1e-3 absolute.  Against exact fp32
attention the FP8 result stays within e4m3 noise (rel L2 <= 0.1).
"""

from __future__ import annotations

import pytest
import torch

import fp8_oracle as oracle

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _qkv(b: int, seq: int, heads: int = 4, seed: int = 0, std: float = 1.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(b, seq, 3 * heads * 64, generator=g) * std).to(torch.bfloat16)


def _rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm()).item()


def _per_part_err(got: torch.Tensor, ref: torch.Tensor, c: int) -> list[float]:
    return [oracle.max_rel_err(got[..., i * c:(i + 1) * c], ref[..., i * c:(i + 1) * c]) for i in range(3)]


@pytest.mark.parametrize("b,seq", [(4, 256), (8, 16), (3, 128), (2, 48), (2, 144), (2, 32)])
def test_attention_forward_matches_oracle(cuda, b, seq):
    from fp8_b200.attention import attention_fwd

    qkv = _qkv(b, seq, seed=seq)
    o, lse, sc = attention_fwd(qkv.to(cuda), 4)
    o_ref, lse_ref, sc_ref = oracle.attention_fwd(qkv, 4)
    assert torch.equal(sc[..., :3].cpu(), sc_ref)
    assert oracle.max_rel_err(o, o_ref) <= TOL
    assert (lse.cpu() - lse_ref).abs().max().item() <= 1e-3
    assert _rel_l2(o.cpu(), oracle.attention_exact(qkv, 4)) <= 0.1


@pytest.mark.parametrize("b,seq", [(4, 256), (8, 16), (2, 144), (2, 48)])
def test_attention_backward_matches_oracle(cuda, b, seq):
    from fp8_b200.attention import attention_bwd, attention_fwd

    qkv = _qkv(b, seq, seed=100 + seq)
    g = torch.Generator().manual_seed(7)
    do = (torch.randn(b, seq, 256, generator=g) * 1e-2).to(torch.bfloat16)
    o, lse, sc = attention_fwd(qkv.to(cuda), 4)
    dqkv = attention_bwd(qkv.to(cuda), o, do.to(cuda), lse, sc, 4)
    ref = oracle.attention_bwd(qkv, o.cpu(), do, lse.cpu(), 4)
    errs = _per_part_err(dqkv.cpu(), ref, 256)
    assert max(errs) <= TOL, errs
    # and the straight-through gradient is that of exact attention up to e4m3 noise
    x = qkv.float().requires_grad_(True)
    xs = x.view(b, seq, 3, 4, 64).permute(2, 0, 3, 1, 4)
    oe = torch.nn.functional.scaled_dot_product_attention(xs[0], xs[1], xs[2]).transpose(1, 2).reshape(b, seq, 256)
    oe.backward(do.float())
    assert _rel_l2(dqkv.cpu(), x.grad) <= 0.1


def test_attention_edge_scales(cuda):
    """One head all zeros (scale 1.0, output 0) and one head with large values."""
    from fp8_b200.attention import attention_fwd

    qkv = _qkv(2, 64, seed=5)
    qkv.view(2, 64, 3, 4, 64)[0, :, :, 1, :] = 0
    qkv.view(2, 64, 3, 4, 64)[1, :, :, 2, :] *= 1000
    o, lse, sc = attention_fwd(qkv.to(cuda), 4)
    o_ref, lse_ref, sc_ref = oracle.attention_fwd(qkv, 4)
    assert torch.equal(sc[..., :3].cpu(), sc_ref)
    assert sc[0, 1, :3].eq(1.0).all()
    assert torch.count_nonzero(o.view(2, 64, 4, 64)[0, :, 1, :]) == 0
    assert oracle.max_rel_err(o, o_ref) <= TOL
    assert torch.isfinite(lse).all()


def test_fp8_attention_autograd_and_full_size(cuda):
    """Autograd through fp8_attention at the UNet's 16x16 size (B = 128, L = 256): finite, and
    on a sample of images equal to the oracle."""
    from fp8_b200.attention import fp8_attention

    qkv = _qkv(128, 256, seed=11).to(cuda).requires_grad_(True)
    o = fp8_attention(qkv, 4)
    g = torch.Generator().manual_seed(12)
    do = (torch.randn(128, 256, 256, generator=g) * 1e-2).to(torch.bfloat16).to(cuda)
    o.backward(do)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and torch.isfinite(qkv.grad).all()
    idx = [0, 63, 127]
    sub = qkv.detach()[idx].cpu()
    o_ref, lse_ref, _ = oracle.attention_fwd(sub, 4)
    assert oracle.max_rel_err(o[idx], o_ref) <= TOL
    ref = oracle.attention_bwd(sub, o[idx].detach().cpu(), do[idx].cpu(), lse_ref, 4)
    assert max(_per_part_err(qkv.grad[idx].cpu(), ref, 256)) <= TOL
