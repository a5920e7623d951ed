"""GPU parity: the tcgen05 3x3 conv (fwd, dX, dW) against the CPU oracle and the reference golden outputs.

Tolerance (the parity contract): max|y - ref| / max|ref| <= 1e-2, where the
reference is fp32 accumulation of the same e4m3 operands times the scales, in bf16.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fp8_oracle as oracle

pytestmark = pytest.mark.gpu

TOL = 1e-2

SUPPORTED = [
    (128, 128, 32, 32),
    (128, 256, 32, 32),
    (256, 256, 16, 16),
    (512, 256, 16, 16),
    (256, 256, 8, 8),
    (512, 256, 8, 8),
    (512, 128, 32, 32),
    (256, 256, 32, 32),
    (256, 256, 4, 4),
]


def _rand_q(shape, seed, device, scale=1.0):
    """Random channels_last bf16 tensor quantised by the oracle -> (fp8 on device, scale on device)."""
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    q, s = oracle.quantize_tensor(x)
    return q.to(device), s.to(device)


def _golden_case(golden, tag, device):
    b, cin, cout, h, w = (int(v) for v in golden[f"{tag}_dims"])

    def fp8(arr, shape):
        return torch.from_numpy(arr.reshape(shape)).view(torch.float8_e4m3fn).permute(0, 3, 1, 2).to(device)

    def bf16(arr, shape):
        return torch.from_numpy(arr.reshape(shape).view(np.int16)).view(torch.bfloat16).permute(0, 3, 1, 2)

    sx, sw, sdy = (torch.tensor(float(v), device=device) for v in golden[f"{tag}_scales"])
    return dict(
        xq=fp8(golden[f"{tag}_xq"], (b, h, w, cin)),
        wq=fp8(golden[f"{tag}_wq"], (cout, 3, 3, cin)),
        dyq=fp8(golden[f"{tag}_dyq"], (b, h, w, cout)),
        sx=sx, sw=sw, sdy=sdy,
        y=bf16(golden[f"{tag}_y"], (b, h, w, cout)),
        dx=bf16(golden[f"{tag}_dx"], (b, h, w, cin)),
        dw=bf16(golden[f"{tag}_dw"], (cout, 3, 3, cin)),
    )


@pytest.mark.parametrize("tag", ["c128x8", "c256x4", "c128to256x16", "c128x32"])
def test_conv_matches_reference_kernel_outputs(cuda, golden, tag):
    from fp8_b200 import ops

    c = _golden_case(golden, tag, cuda)
    y = ops.conv3x3_fwd(c["xq"], c["wq"], c["sx"], c["sw"])
    dx = ops.conv3x3_dgrad(c["dyq"], c["wq"], c["sdy"], c["sw"])
    dw = ops.conv3x3_wgrad(c["xq"], c["dyq"], c["sx"], c["sdy"])
    assert y.is_contiguous(memory_format=torch.channels_last)
    assert oracle.max_rel_err(y, c["y"]) <= TOL
    assert oracle.max_rel_err(dx, c["dx"]) <= TOL
    assert oracle.max_rel_err(dw, c["dw"]) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("cin,cout,h,w", SUPPORTED)
def test_conv_fwd_all_unet_shapes(cuda, cin, cout, h, w):
    from fp8_b200 import ops

    b = max(2, 256 // (h * w))
    xq, sx = _rand_q((b, cin, h, w), seed=cin + cout + h, device=cuda)
    wq, sw = _rand_q((cout, cin, 3, 3), seed=7 + cin, device=cuda, scale=0.05)
    y = ops.conv3x3_fwd(xq, wq, sx, sw)
    ref = oracle.conv_fwd(xq.cpu(), wq.cpu(), sx.item(), sw.item())
    assert oracle.max_rel_err(y, ref) <= TOL


@pytest.mark.parametrize("cin,cout,h,w", SUPPORTED)
def test_conv_dgrad_all_unet_shapes(cuda, cin, cout, h, w):
    from fp8_b200 import ops

    b = max(2, 256 // (h * w))
    dyq, sdy = _rand_q((b, cout, h, w), seed=cin * 3 + cout + h, device=cuda, scale=1e-2)
    wq, sw = _rand_q((cout, cin, 3, 3), seed=9 + cin, device=cuda, scale=0.05)
    dx = ops.conv3x3_dgrad(dyq, wq, sdy, sw)
    ref = oracle.conv_dx(dyq.cpu(), wq.cpu(), sdy.item(), sw.item())
    assert oracle.max_rel_err(dx, ref) <= TOL


@pytest.mark.parametrize("cin,cout,h,w", SUPPORTED)
def test_conv_wgrad_all_unet_shapes(cuda, cin, cout, h, w):
    from fp8_b200 import ops

    b = max(2, 512 // (h * w))
    xq, sx = _rand_q((b, cin, h, w), seed=cin + 5 * cout + h, device=cuda)
    dyq, sdy = _rand_q((b, cout, h, w), seed=cin + 7 * cout + w, device=cuda, scale=1e-2)
    dw = ops.conv3x3_wgrad(xq, dyq, sx, sdy)
    ref = oracle.conv_dw(xq.cpu(), dyq.cpu(), sx.item(), sdy.item())
    assert dw.shape == (cout, cin, 3, 3) and dw.is_contiguous(memory_format=torch.channels_last)
    assert oracle.max_rel_err(dw, ref) <= TOL


@pytest.mark.parametrize("cin,cout,h,w", [(128, 128, 32, 32), (256, 256, 8, 8), (512, 256, 16, 16)])
def test_conv_wgrad_widened_fp32(cuda, cin, cout, h, w):
    """widen=True: fp32 dW holding bf16 values (what autograd stores for an fp32 weight), equal to
    the bf16 result widened up to the unordered split-K additions (one bf16 step), and within the
    oracle tolerance."""
    from fp8_b200 import ops

    b = max(2, 2048 // (h * w))
    xq, sx = _rand_q((b, cin, h, w), seed=cin + h, device=cuda)
    dyq, sdy = _rand_q((b, cout, h, w), seed=cout + w + 1, device=cuda, scale=1e-2)
    dw32 = ops.conv3x3_wgrad(xq, dyq, sx, sdy, 0, True)
    dw16 = ops.conv3x3_wgrad(xq, dyq, sx, sdy)
    assert dw32.dtype == torch.float32 and dw32.is_contiguous(memory_format=torch.channels_last)
    assert torch.equal(dw32.bfloat16().float(), dw32)  # bf16 values
    ref16 = dw16.float()
    assert ((dw32 - ref16).abs() <= 2.0 ** -7 * ref16.abs() + 1e-4 * ref16.abs().max()).all()
    ref = oracle.conv_dw(xq.cpu(), dyq.cpu(), sx.item(), sdy.item())
    assert oracle.max_rel_err(dw32, ref) <= TOL


def test_batched_weight_relayout_gives_the_same_dgrad(cuda):
    """transpose_conv_weights (one launch for many weights) + conv3x3_dgrad_pre equal conv3x3_dgrad, which
    re-lays each weight out itself, bit for bit, for the shapes whose data-grad does not read in place."""
    from fp8_b200 import ops

    shapes = [(256, 256, 8, 8), (512, 256, 8, 8), (256, 256, 4, 4), (256, 512, 4, 4), (128, 256, 16, 16)]
    cases = []
    for i, (cin, cout, h, w) in enumerate(shapes):
        b = 16
        wq, sw = _rand_q((cout, cin, 3, 3), seed=40 + i, device=cuda, scale=0.05)
        dyq, sdy = _rand_q((b, cout, h, w), seed=50 + i, device=cuda, scale=1e-2)
        cases.append((cin, cout, h, w, b, wq, sw, dyq, sdy))
    need = [c for c in cases if ops.dgrad_needs_relayout(c[4], c[2], c[3], c[0], c[1])]
    assert len(need) >= 3
    wts = ops.transpose_conv_weights([c[5] for c in need])
    for (cin, cout, h, w, b, wq, sw, dyq, sdy), wq_t in zip(need, wts):
        assert wq_t.shape == (cin, 9 * cout)
        assert torch.equal(ops.conv3x3_dgrad_pre(dyq, wq_t, sdy, sw), ops.conv3x3_dgrad(dyq, wq, sdy, sw))


@pytest.mark.parametrize("split_k", [1, 3, 7])
def test_conv_wgrad_split_counts(cuda, split_k):
    from fp8_b200 import ops

    xq, sx = _rand_q((8, 128, 16, 16), seed=21, device=cuda)
    dyq, sdy = _rand_q((8, 128, 16, 16), seed=22, device=cuda, scale=1e-2)
    dw = ops.conv3x3_wgrad(xq, dyq, sx, sdy, split_k)
    ref = oracle.conv_dw(xq.cpu(), dyq.cpu(), sx.item(), sdy.item())
    assert oracle.max_rel_err(dw, ref) <= TOL


@pytest.mark.parametrize("epilogue", [1, 2])
def test_conv_fwd_bias_silu_epilogue(cuda, epilogue):
    from fp8_b200 import ops

    xq, sx = _rand_q((4, 128, 32, 32), seed=31, device=cuda)
    wq, sw = _rand_q((128, 128, 3, 3), seed=32, device=cuda, scale=0.05)
    g = torch.Generator().manual_seed(33)
    bias = (torch.randn(128, generator=g) * 0.1).to(torch.bfloat16)
    y = ops.conv3x3_fwd(xq, wq, sx, sw, bias.to(cuda), epilogue)
    ref = oracle.conv_fwd(xq.cpu(), wq.cpu(), sx.item(), sw.item(), bias=bias, silu=(epilogue == 2))
    assert oracle.max_rel_err(y, ref) <= TOL


@pytest.mark.parametrize("bm_sub,bn", [(2, 128), (1, 64), (1, 128)])
def test_conv_fwd_tile_variants(cuda, bm_sub, bn):
    from fp8_b200 import _lib, ops

    xq, sx = _rand_q((8, 128, 32, 32), seed=41, device=cuda)
    wq, sw = _rand_q((128, 128, 3, 3), seed=42, device=cuda, scale=0.05)
    ref = oracle.conv_fwd(xq.cpu(), wq.cpu(), sx.item(), sw.item())
    try:
        _lib.set_tile_override(bm_sub, bn, 0)
        y = ops.conv3x3_fwd(xq, wq, sx, sw)
    finally:
        _lib.set_tile_override(0, 0, 0)
    assert oracle.max_rel_err(y, ref) <= TOL


@pytest.mark.parametrize("group", [1, 3])
def test_conv_wgrad_group_variants(cuda, group):
    from fp8_b200 import _lib, ops

    xq, sx = _rand_q((4, 128, 32, 32), seed=51, device=cuda)
    dyq, sdy = _rand_q((4, 128, 32, 32), seed=52, device=cuda, scale=1e-2)
    ref = oracle.conv_dw(xq.cpu(), dyq.cpu(), sx.item(), sdy.item())
    try:
        _lib.set_tile_override(0, 0, group)
        dw = ops.conv3x3_wgrad(xq, dyq, sx, sdy)
    finally:
        _lib.set_tile_override(0, 0, 0)
    assert oracle.max_rel_err(dw, ref) <= TOL


def test_conv_config2_full_size(cuda):
    """BASELINE config 2 at full size: B=128, 128->128, 32x32 (M=131072, N=128, K=1152)."""
    from fp8_b200 import ops

    xq, sx = _rand_q((128, 128, 32, 32), seed=0, device=cuda)
    wq, sw = _rand_q((128, 128, 3, 3), seed=1, device=cuda, scale=0.05)
    y = ops.conv3x3_fwd(xq, wq, sx, sw)
    ref = oracle.conv_fwd(xq.cpu(), wq.cpu(), sx.item(), sw.item())
    assert oracle.max_rel_err(y, ref) <= TOL
    assert ops.device_error() == 0


HALO_SHAPES = [s for s in SUPPORTED if s[3] in (16, 32)]


@pytest.mark.parametrize("algo", [1, 2, 3, 4])
@pytest.mark.parametrize("cin,cout,h,w", HALO_SHAPES)
def test_conv_fwd_and_dgrad_every_algorithm(cuda, algo, cin, cout, h, w):
    """Tap-by-tap GEMM (algo 1), the single-CTA halo kernel (algo 2), the
    CTA-pair halo kernel (algo 3) and the transposed halo kernel (algo 4; both
    where the reduced dimension is 128 channels) against the oracle."""
    from fp8_b200 import _lib, ops

    b = 2 if h == 32 else 4
    xq, sx = _rand_q((b, cin, h, w), seed=3 * cin + cout + w, device=cuda)
    dyq, sdy = _rand_q((b, cout, h, w), seed=5 * cin + cout + h, device=cuda, scale=1e-2)
    wq, sw = _rand_q((cout, cin, 3, 3), seed=11 + cout, device=cuda, scale=0.05)
    y_ref = oracle.conv_fwd(xq.cpu(), wq.cpu(), sx.item(), sw.item())
    dx_ref = oracle.conv_dx(dyq.cpu(), wq.cpu(), sdy.item(), sw.item())
    try:
        _lib.set_conv_algo(algo)
        y = ops.conv3x3_fwd(xq, wq, sx, sw)
        dx = ops.conv3x3_dgrad(dyq, wq, sdy, sw)
    finally:
        _lib.set_conv_algo(0)
    assert oracle.max_rel_err(y, y_ref) <= TOL
    assert oracle.max_rel_err(dx, dx_ref) <= TOL
    assert ops.device_error() == 0


def test_conv_halo_bias_silu_epilogue(cuda):
    from fp8_b200 import ops

    xq, sx = _rand_q((2, 128, 16, 16), seed=61, device=cuda)
    wq, sw = _rand_q((256, 128, 3, 3), seed=62, device=cuda, scale=0.05)
    g = torch.Generator().manual_seed(63)
    bias = (torch.randn(256, generator=g) * 0.1).to(torch.bfloat16)
    y = ops.conv3x3_fwd(xq, wq, sx, sw, bias.to(cuda), 2)
    ref = oracle.conv_fwd(xq.cpu(), wq.cpu(), sx.item(), sw.item(), bias=bias, silu=True)
    assert oracle.max_rel_err(y, ref) <= TOL


@pytest.mark.parametrize("algo", [2, 3, 4])
def test_conv_config2_halo_variants_full_size(cuda, algo):
    """Config 2 at full size through both halo kernels, fwd and data-grad."""
    from fp8_b200 import _lib, ops

    xq, sx = _rand_q((128, 128, 32, 32), seed=70, device=cuda)
    dyq, sdy = _rand_q((128, 128, 32, 32), seed=71, device=cuda, scale=1e-2)
    wq, sw = _rand_q((128, 128, 3, 3), seed=72, device=cuda, scale=0.05)
    try:
        _lib.set_conv_algo(algo)
        y = ops.conv3x3_fwd(xq, wq, sx, sw)
        dx = ops.conv3x3_dgrad(dyq, wq, sdy, sw)
    finally:
        _lib.set_conv_algo(0)
    assert oracle.max_rel_err(y, oracle.conv_fwd(xq.cpu(), wq.cpu(), sx.item(), sw.item())) <= TOL
    assert oracle.max_rel_err(dx, oracle.conv_dx(dyq.cpu(), wq.cpu(), sdy.item(), sw.item())) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("cin,cout", [(128, 128), (128, 256), (512, 128)])
def test_conv_transposed_halo_tail_half_tiles(cuda, cin, cout):
    """B = 40 at 32x32: 160 tiles of 256 pixels per column tile, more than one
    round of the persistent grid, so the last tiles run as 128-pixel halves."""
    from fp8_b200 import ops

    xq, sx = _rand_q((40, cin, 32, 32), seed=81 + cout, device=cuda)
    dyq, sdy = _rand_q((40, cout, 32, 32), seed=82 + cin, device=cuda, scale=1e-2)
    wq, sw = _rand_q((cout, cin, 3, 3), seed=83, device=cuda, scale=0.05)
    y = ops.conv3x3_fwd(xq, wq, sx, sw)
    dx = ops.conv3x3_dgrad(dyq, wq, sdy, sw)
    assert oracle.max_rel_err(y, oracle.conv_fwd(xq.cpu(), wq.cpu(), sx.item(), sw.item())) <= TOL
    assert oracle.max_rel_err(dx, oracle.conv_dx(dyq.cpu(), wq.cpu(), sdy.item(), sw.item())) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("algo", [1, 0])
@pytest.mark.parametrize("cin,cout,h,w", HALO_SHAPES)
def test_conv_wgrad_tap_and_halo_paths(cuda, algo, cin, cout, h, w):
    """Weight gradient with per-tap X windows (algo 1) and with one halo box per
    column tap (the default for 32x32 and 16x16 images) against the oracle."""
    from fp8_b200 import _lib, ops

    b = 2 if h == 32 else 4
    xq, sx = _rand_q((b, cin, h, w), seed=7 * cin + cout + h, device=cuda)
    dyq, sdy = _rand_q((b, cout, h, w), seed=9 * cin + cout + w, device=cuda, scale=1e-2)
    ref = oracle.conv_dw(xq.cpu(), dyq.cpu(), sx.item(), sdy.item())
    try:
        _lib.set_conv_algo(algo)
        dw = ops.conv3x3_wgrad(xq, dyq, sx, sdy)
    finally:
        _lib.set_conv_algo(0)
    assert oracle.max_rel_err(dw, ref) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("cin,h,w,b", [(128, 32, 32, 2), (256, 32, 32, 40), (256, 16, 16, 8), (512, 16, 16, 4)])
def test_dgrad_reads_forward_weights_in_place(cuda, cin, h, w, b):
    """Cout = 128: the transposed halo kernel takes the forward's weights
    [Cout][3][3][Cin] as an MN-major operand.  Same products in the same order as
    the re-laid-out [Cin][3][3][Cout] path, so the results are bit-identical."""
    from ctypes import c_void_p

    from fp8_b200 import _lib, ops

    cout = 128
    lib = _lib.load()
    assert lib.fp8_conv3x3_dgrad_w_workspace_bytes(b, h, w, cin, cout) == 0
    dyq, sdy = _rand_q((b, cout, h, w), seed=91 + cin, device=cuda, scale=1e-2)
    wq, sw = _rand_q((cout, cin, 3, 3), seed=92 + h, device=cuda, scale=0.05)
    p = lambda t: c_void_p(t.data_ptr())  # noqa: E731
    st = c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    dx = ops.conv3x3_dgrad(dyq, wq, sdy, sw)
    wt = torch.empty((cin, 9 * cout), device=cuda, dtype=torch.float8_e4m3fn)
    _lib.call("fp8_conv_weight_transpose", p(wq), p(wt), cout, cin, st)
    dx2 = torch.empty_like(dx)
    _lib.call("fp8_conv3x3_dgrad", p(dyq), p(wt), p(dx2), p(sdy), p(sw), b, h, w, cin, cout, st)
    torch.cuda.synchronize()
    assert torch.equal(dx.view(torch.int16), dx2.view(torch.int16))
    assert oracle.max_rel_err(dx, oracle.conv_dx(dyq.cpu(), wq.cpu(), sdy.item(), sw.item())) <= TOL
    assert ops.device_error() == 0


def test_dgrad_w_workspace_path(cuda):
    """Cout = 256: the weights are re-laid out into the caller's workspace first."""
    from fp8_b200 import _lib, ops

    b, cin, cout, h, w = 2, 128, 256, 32, 32
    assert _lib.load().fp8_conv3x3_dgrad_w_workspace_bytes(b, h, w, cin, cout) == 9 * cin * cout
    dyq, sdy = _rand_q((b, cout, h, w), seed=95, device=cuda, scale=1e-2)
    wq, sw = _rand_q((cout, cin, 3, 3), seed=96, device=cuda, scale=0.05)
    dx = ops.conv3x3_dgrad(dyq, wq, sdy, sw)
    assert oracle.max_rel_err(dx, oracle.conv_dx(dyq.cpu(), wq.cpu(), sdy.item(), sw.item())) <= TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("mode", [1, 2])
def test_launch_modes_give_the_same_results(cuda, mode):
    """Programmatic dependent launch only changes when CTAs may start: a
    quantize -> fwd -> quantize -> dX -> dW chain gives the same bytes as plain
    stream order (dW up to the order of its fp32 split-K additions, i.e. one
    bf16 rounding step)."""
    from fp8_b200 import _lib, ops

    g = torch.Generator().manual_seed(123)
    x = torch.randn(8, 128, 32, 32, generator=g).to(torch.bfloat16).to(cuda).contiguous(
        memory_format=torch.channels_last)
    w = (torch.randn(128, 128, 3, 3, generator=g) * 0.05).to(torch.bfloat16).to(cuda).contiguous(
        memory_format=torch.channels_last)
    dy = (torch.randn(8, 128, 32, 32, generator=g) * 1e-2).to(torch.bfloat16).to(cuda).contiguous(
        memory_format=torch.channels_last)

    def chain():
        xq, sx, wq, sw = ops.quantize_current_pair(x, w)
        y = ops.conv3x3_fwd(xq, wq, sx, sw)
        dyq, sdy = ops.quantize_current(dy)
        dx = ops.conv3x3_dgrad(dyq, wq, sdy, sw)
        dw = ops.conv3x3_wgrad(xq, dyq, sx, sdy)
        torch.cuda.synchronize()
        return dict(xq=xq.view(torch.uint8), sx=sx, y=y, dyq=dyq.view(torch.uint8), sdy=sdy, dx=dx, dw=dw)

    ref = chain()
    try:
        _lib.set_pdl(mode)
        got = chain()
    finally:
        _lib.set_pdl(0)
    for k in ("xq", "sx", "y", "dyq", "sdy", "dx"):
        assert torch.equal(ref[k], got[k]), k
    a, b = ref["dw"].float(), got["dw"].float()
    excess = (a - b).abs() - (2.0 ** -7 * a.abs() + 1e-4 * a.abs().max())
    assert excess.max().item() <= 0.0, excess.max().item()
    assert ops.device_error() == 0


@pytest.mark.parametrize("fused", [True, False])
def test_wgrad_conversion_fused_and_separate_agree(cuda, fused):
    """The weight gradient with the accumulator conversion folded into the split-K launch
    (cooperative, grid barrier) and as a separate launch: the oracle's dW, bf16 and widened fp32,
    eagerly and from a CUDA graph."""
    from fp8_b200 import _lib, ops

    g = torch.Generator().manual_seed(41)
    x = (torch.randn(32, 128, 32, 32, generator=g)).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    dy = (torch.randn(32, 128, 32, 32, generator=g) * 1e-2).to(torch.bfloat16).contiguous(
        memory_format=torch.channels_last)
    xq, sx = oracle.quantize_tensor(x)
    dyq, sdy = oracle.quantize_tensor(dy)
    ref = oracle.conv_dw(xq, dyq, sx, sdy)
    try:
        _lib.set_wgrad_fused(fused)
        args = (xq.to(cuda), dyq.to(cuda), sx.to(cuda), sdy.to(cuda))
        dw = ops.conv3x3_wgrad(*args, 0)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            ops.conv3x3_wgrad(*args, 0)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            dw_g = ops.conv3x3_wgrad(*args, 0)
        graph.replay()
        graph.replay()
        torch.cuda.synchronize()
    finally:
        _lib.set_wgrad_fused(False)
    assert oracle.max_rel_err(dw, ref) <= TOL
    assert oracle.max_rel_err(dw_g, ref) <= TOL
    assert _lib.device_error() == 0


@pytest.mark.parametrize("cin,cout,h,w", [(128, 128, 32, 32), (256, 256, 8, 8), (512, 256, 16, 16)])
def test_conv3x3_backward_overlapped_matches_separate_ops(cuda, cin, cout, h, w):
    """conv3x3_backward (dW on a side stream beside dX) gives conv3x3_dgrad's dx bit for bit and
    conv3x3_wgrad's dw within the oracle tolerance, eagerly, widened to fp32, with pre-transposed
    weights, and replayed from a CUDA graph (the fork and join are captured)."""
    from fp8_b200 import ops

    b = 4
    xq, sx = _rand_q((b, cin, h, w), seed=301 + cin, device=cuda)
    dyq, sdy = _rand_q((b, cout, h, w), seed=302 + cout, device=cuda, scale=1e-2)
    wq, sw = _rand_q((cout, cin, 3, 3), seed=303 + h, device=cuda, scale=0.05)
    dx_ref = ops.conv3x3_dgrad(dyq, wq, sdy, sw)
    dw_oracle = oracle.conv_dw(xq.cpu(), dyq.cpu(), sx.item(), sdy.item())
    dx, dw = ops.conv3x3_backward(dyq, wq, sdy, sw, xq, sx)
    torch.cuda.synchronize()
    assert torch.equal(dx.view(torch.int16), dx_ref.view(torch.int16))
    assert dw.dtype == torch.bfloat16 and dw.is_contiguous(memory_format=torch.channels_last)
    assert oracle.max_rel_err(dw, dw_oracle) <= TOL
    _, dw32 = ops.conv3x3_backward(dyq, wq, sdy, sw, xq, sx, 0, True)
    assert dw32.dtype == torch.float32 and oracle.max_rel_err(dw32, dw_oracle) <= TOL
    wq_t = ops.transpose_conv_weights([wq])[0]
    dx_pre, _ = ops.conv3x3_backward(dyq, wq, sdy, sw, xq, sx, 0, False, wq_t)
    assert torch.equal(dx_pre.view(torch.int16), ops.conv3x3_dgrad_pre(dyq, wq_t, sdy, sw).view(torch.int16))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        ops.conv3x3_backward(dyq, wq, sdy, sw, xq, sx)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        gdx, gdw = ops.conv3x3_backward(dyq, wq, sdy, sw, xq, sx)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(gdx.view(torch.int16), dx_ref.view(torch.int16))
    assert oracle.max_rel_err(gdw, dw_oracle) <= TOL
    assert ops.device_error() == 0
