"""GPU parity: the scaled FP8 linear (tcgen05 GEMM) against the CPU oracle.

BASELINE config 1 (X [4096,512], W [512,2048], bias) and config 3 (tokens
[32768,256], qkv W [256,768], out W [256,256]).  Tolerance: max relative error
1e-2 against fp32 accumulation of the same e4m3 operands, bf16 output.
"""

from __future__ import annotations

import pytest
import torch

import fp8_oracle as oracle

pytestmark = pytest.mark.gpu

TOL = 1e-2


def _q2d(shape, seed, device, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16)
    q, s = oracle.quantize_tensor(x)
    return x, q.to(device), s.to(device)


@pytest.mark.parametrize(
    "m,k,n,epilogue",
    [
        (4096, 512, 2048, 1),  # config 1 with bias
        (4096, 512, 2048, 0),
        (32768, 256, 768, 0),  # config 3 qkv
        (32768, 256, 256, 0),  # config 3 out
        (128, 512, 512, 2),  # time-embedding MLP shape, bias + SiLU
        (100, 128, 96, 0),  # ragged M, N not a multiple of 64
        (1, 64, 32, 0),
    ],
)
def test_gemm_matches_oracle(cuda, m, k, n, epilogue):
    from fp8_b200 import ops

    _, aq, sa = _q2d((m, k), seed=m + k, device=cuda)
    _, bq, sb = _q2d((n, k), seed=n + 3, device=cuda, scale=0.02)
    g = torch.Generator().manual_seed(n)
    bias = (torch.randn(n, generator=g) * 0.01).to(torch.bfloat16)
    y = ops.gemm(aq, bq, sa, sb, bias.to(cuda) if epilogue else None, epilogue)
    ref = oracle.linear_fwd(aq.cpu(), bq.cpu(), sa.item(), sb.item(), bias=bias if epilogue else None,
                            silu=epilogue == 2)
    assert y.shape == (m, n)
    assert oracle.max_rel_err(y, ref) <= TOL


@pytest.mark.parametrize("m,n,k", [(4096, 2048, 512), (32768, 768, 256), (300, 256, 128)])
def test_gemm_wgrad_matches_oracle(cuda, m, n, k):
    from fp8_b200 import ops

    _, dyq, sdy = _q2d((m, n), seed=m + n, device=cuda, scale=1e-2)
    _, xq, sx = _q2d((m, k), seed=k + 1, device=cuda)
    dw = ops.gemm_wgrad(dyq, xq, sdy, sx)
    ref = oracle.linear_dw(dyq.cpu(), xq.cpu(), sdy.item(), sx.item())
    assert dw.shape == (n, k)
    assert oracle.max_rel_err(dw, ref) <= TOL


def test_fp8_linear_autograd_matches_oracle(cuda):
    from fp8_b200.linear import fp8_linear

    g = torch.Generator().manual_seed(0)
    x = torch.randn(4096, 512, generator=g).to(torch.bfloat16)
    w_math = (torch.randn(512, 2048, generator=g) * 0.02).to(torch.bfloat16)  # config-1 W [in, out]
    w = w_math.t().contiguous()  # nn.Linear layout [out, in]
    b = (torch.randn(2048, generator=g) * 0.01).to(torch.bfloat16)
    dy = (torch.randn(4096, 2048, generator=g) * 1e-2).to(torch.bfloat16)

    xd = x.to(cuda).requires_grad_(True)
    wd = w.to(cuda).requires_grad_(True)
    bd = b.to(cuda).requires_grad_(True)
    y = fp8_linear(xd, wd, bd)
    y.backward(dy.to(cuda))

    xq, sx = oracle.quantize_tensor(x)
    wq, sw = oracle.quantize_tensor(w)
    dyq, sdy = oracle.quantize_tensor(dy)
    assert oracle.max_rel_err(y, oracle.linear_fwd(xq, wq, sx, sw, bias=b)) <= TOL
    assert oracle.max_rel_err(xd.grad, oracle.linear_dx(dyq, wq, sdy, sw)) <= TOL
    assert oracle.max_rel_err(wd.grad, oracle.linear_dw(dyq, xq, sdy, sx)) <= TOL
    assert oracle.max_rel_err(bd.grad, dy.float().sum(0)) <= TOL
