"""GPU check: the fused clip + AdamW + EMA step (fp8_b200.optim.FusedAdamWEMA) against
torch's clip_grad_norm_, torch.optim.AdamW and the foreach EMA of the training step,
over several steps with clipping active and inactive.

Tolerance: max|got - ref| / max|ref| <= 1e-5 per tensor (same fp32 formulas, the
order of a few roundings differs)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("max_norm", [1.0, 1e4, None])
def test_fused_adamw_ema_matches_torch(cuda, max_norm):
    from fp8_b200.optim import FusedAdamWEMA

    g = torch.Generator().manual_seed(0)
    shapes = [(256, 128, 3, 3), (512,), (77, 13), (3, 5, 7, 9), (4096, 64)] + [(100,)] * 50  # > one launch group
    base = [torch.randn(*s, generator=g) * 0.1 for s in shapes]
    grads = [[torch.randn(*s, generator=g) * 0.05 for s in shapes] for _ in range(4)]

    def params():
        ps = []
        for b in base:
            p = b.clone().to(cuda)
            if p.dim() == 4:
                p = p.contiguous(memory_format=torch.channels_last)
            ps.append(torch.nn.Parameter(p))
        return ps

    pa, pb = params(), params()
    ema_a = [p.detach().clone() for p in pa]
    ema_b = [p.detach().clone() for p in pb]
    opt_a = FusedAdamWEMA(pa, lr=2e-4, max_grad_norm=max_norm, ema=ema_a, ema_beta=0.99)
    opt_b = torch.optim.AdamW(pb, lr=2e-4, fused=True)
    for step_grads in grads:
        for p, q, gr in zip(pa, pb, step_grads):
            p.grad = gr.to(cuda).contiguous(memory_format=torch.channels_last) if p.dim() == 4 else gr.to(cuda)
            q.grad = p.grad.clone()
        opt_a.step()
        if max_norm is not None:
            torch.nn.utils.clip_grad_norm_(pb, max_norm=max_norm)
        opt_b.step()
        with torch.no_grad():
            torch._foreach_mul_(ema_b, 0.99)
            torch._foreach_add_(ema_b, [p.detach() for p in pb], alpha=0.01)
    torch.cuda.synchronize()
    assert opt_a.step_count.item() == 4.0
    for x, y in zip(pa + ema_a, pb + ema_b):
        d = (x.detach() - y.detach()).abs().max() / y.detach().abs().max()
        assert d.item() <= 1e-5
