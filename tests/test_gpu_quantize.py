"""GPU parity: quantize kernels are bit-exact (bytes and scales) against the CPU oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fp8_oracle as oracle

pytestmark = pytest.mark.gpu


def _bytes(t: torch.Tensor) -> np.ndarray:
    """float8 tensor -> bytes in memory order."""
    t = t.detach()
    flat = t.as_strided((t.numel(),), (1,)) if t.is_contiguous() or t.is_contiguous(
        memory_format=torch.channels_last) else t.reshape(-1)
    return flat.view(torch.uint8).cpu().numpy()


def _check_current(x: torch.Tensor):
    from fp8_b200 import ops

    q, s = ops.quantize_current(x)
    q_ref, s_ref = oracle.quantize_current(x.cpu())
    assert q.dtype == torch.float8_e4m3fn and q.stride() == x.stride()
    assert np.float32(s.item()).tobytes() == s_ref.tobytes(), (s.item(), s_ref)
    got = _bytes(q)
    if not np.array_equal(got, q_ref):
        bad = np.nonzero(got != q_ref)[0]
        raise AssertionError(f"{bad.size} byte mismatches, first at {bad[:5]}: {got[bad[:5]]} vs {q_ref[bad[:5]]}")


def _gen(shape, seed, scale=1.0, device="cuda"):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).to(device)


@pytest.mark.parametrize(
    "shape,scale",
    [
        ((2, 3, 4, 5), 1.0),
        ((1, 1, 1, 1), 3.0),
        ((3, 5, 7, 11), 1.0),  # n % 8 != 0: scalar tail
        ((1, 1, 1, 8192 + 13), 37.0),
        ((128, 128, 32, 32), 1.0),  # config-2 activation, 16.7M elements
        ((4, 256, 16, 16), 1e-3),  # small magnitudes: subnormal e4m3 outputs
        ((2, 64, 8, 8), 5e4),  # large magnitudes
    ],
)
def test_quantize_current_bit_exact(cuda, shape, scale):
    _check_current(_gen(shape, seed=hash(shape) & 0xFFFF, scale=scale))


def test_quantize_current_channels_last_keeps_layout(cuda):
    x = _gen((8, 128, 16, 16), seed=3).contiguous(memory_format=torch.channels_last)
    _check_current(x)


def test_quantize_zero_tensor_scale_one(cuda):
    from fp8_b200 import ops

    q, s = ops.quantize_current(torch.zeros(2, 3, 4, 5, dtype=torch.bfloat16, device=cuda))
    assert s.item() == 1.0 and not _bytes(q).any()


def test_quantize_power_of_two_amax_and_ties(cuda):
    # amax exactly 448 * 2**-3 -> scale 2**-3 exactly; values on e4m3 midpoints tie to even
    vals = torch.from_numpy(np.arange(256, dtype=np.uint8)).view(torch.float8_e4m3fn).float()
    fin = torch.unique(vals[torch.isfinite(vals)])
    mids = (fin[1:] + fin[:-1]) / 2 / 8.0  # scaled by the scale 2**-3
    x = torch.cat([mids, fin / 8.0, torch.tensor([56.0])]).to(torch.bfloat16)  # 448/8 = 56 sets amax
    _check_current(x.reshape(1, 1, 1, -1).to(cuda))


def test_quantize_unaligned_view_scalar_path(cuda):
    base = _gen((1, 1, 1, 4099), seed=11)
    x = base[..., 1:]  # 2-byte offset: not 16-byte aligned
    assert x.data_ptr() % 16 != 0
    _check_current(x.contiguous() if not x.is_contiguous() else x)


@pytest.mark.parametrize("prev", [0.05, 1.0, 1e-4, 0.0])
def test_quantize_delayed_bit_exact(cuda, prev):
    from fp8_b200 import ops

    x = _gen((16, 128, 8, 8), seed=5)
    prev_t = torch.tensor(prev, dtype=torch.float32, device=cuda)
    q, s_curr = ops.quantize_delayed(x, prev_t)
    q_ref, s_ref = oracle.quantize_delayed(x.cpu(), prev)
    assert np.float32(s_curr.item()).tobytes() == s_ref.tobytes()
    assert np.array_equal(_bytes(q), q_ref)


@pytest.mark.parametrize(
    "scale",
    [1.0, 0.125, 0.1, 1.0 / 3.0, 0.7071068, 3.0, 7.3e-5, 1.2345678e-2, 2.9e5, 1e30,
     2.0**-60, 2.0**100,  # edges of the fp32 correction-step window
     1e-30, 2.0**-61, 3e30, 1e-40],  # outside it: the double-reciprocal path
)
@pytest.mark.parametrize("offset", [0, 1])  # 1: a view 2 bytes off 16-byte alignment (scalar kernels)
def test_quantize_cast_every_bf16_value(cuda, scale, offset):
    """Every one of the 65,536 bf16 bit patterns (NaN, inf, subnormals included), cast
    with a fixed scale, gives the oracle's byte: both of the GPU's divide-free
    quotients must equal IEEE fp32 division for every input, in the streaming and
    in the scalar kernels."""
    from fp8_b200 import ops

    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.int16)
    buf = torch.zeros(65536 + offset, dtype=torch.int16)
    buf[offset:] = torch.from_numpy(bits.copy())
    x = buf.to(cuda).view(torch.bfloat16)[offset:]
    assert (x.data_ptr() % 16 == 0) == (offset == 0)
    s32 = np.float32(scale)
    q, _ = ops.quantize_delayed(x, torch.tensor(float(s32), dtype=torch.float32, device=cuda))
    q_ref = oracle.cast_with_scale(oracle.bf16_bits_to_f32(bits.view(np.uint16)), s32)
    got = _bytes(q)
    bad = np.nonzero(got != q_ref)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first bf16 bits {bits.view(np.uint16)[bad[:5]]}"


def test_quantize_delayed_ragged(cuda):
    from fp8_b200 import ops

    x = _gen((1, 3, 7, 13), seed=9, scale=20.0)
    prev_t = torch.tensor(0.01, dtype=torch.float32, device=cuda)
    q, s_curr = ops.quantize_delayed(x, prev_t)
    q_ref, s_ref = oracle.quantize_delayed(x.cpu(), 0.01)
    assert np.float32(s_curr.item()).tobytes() == s_ref.tobytes()
    assert np.array_equal(_bytes(q), q_ref)


@pytest.mark.parametrize("name", ["randn", "zeros", "pow2", "ragged", "tiny"])
def test_quantize_matches_golden_scales(cuda, golden, name):
    from fp8_b200 import ops

    bits = golden[f"q_{name}_x"]
    shape = tuple(int(v) for v in golden[f"q_{name}_shape"])
    x = torch.from_numpy(bits.view(np.int16).reshape(shape)).view(torch.bfloat16).to(cuda)
    _, s = ops.quantize_current(x)
    assert np.float32(s.item()).tobytes() == golden[f"q_{name}_scale"].tobytes()
    prev = torch.tensor(float(golden[f"q_{name}_delayed_prev"][0]), device=cuda)
    _, s_curr = ops.quantize_delayed(x, prev)
    assert np.float32(s_curr.item()).tobytes() == golden[f"q_{name}_delayed_scale"].tobytes()


def test_transpose_2d_matches_reference_fixture(cuda, golden):
    from fp8_b200 import ops

    for tag in ("c128x8", "c256x4", "c128to256x16", "c128x32"):
        b, cin, cout, h, w = (int(v) for v in golden[f"{tag}_dims"])
        dyq = torch.from_numpy(golden[f"{tag}_dyq"].reshape(b * h * w, cout)).view(torch.float8_e4m3fn).to(cuda)
        t = ops.transpose_2d(dyq)
        assert np.array_equal(t.view(torch.uint8).cpu().numpy(), golden[f"{tag}_dyt"])


def test_no_device_error_recorded(cuda):
    from fp8_b200 import ops

    assert ops.device_error() == 0


def test_quantize_current_large_tensor(cuda):
    """67 MB of bf16 (the largest UNet activation): about 14 chunks per CTA in each pass."""
    _check_current(_gen((128, 256, 32, 32), seed=21, scale=2.0).contiguous(memory_format=torch.channels_last))


@pytest.mark.parametrize("shape", [(128, 128, 32, 32), (3, 5, 7, 11), (1, 1, 1, 8192 + 13)])
def test_quantize_current_grid_override(cuda, shape):
    """Other grid sizes of the two passes, selected through the tuning override (the
    resident launch off, so that large tensors take the two passes too)."""
    from fp8_b200 import _lib

    try:
        _lib.set_quantize_resident(False)
        _lib.set_quantize_override(1, 3)
        _check_current(_gen(shape, seed=sum(shape), scale=3.0))
    finally:
        _lib.set_quantize_override(0, 0)
        _lib.set_quantize_resident(True)


def test_quantize_current_captured_in_cuda_graph(cuda):
    """Captured in a CUDA graph and replayed on new data: same bytes as the oracle."""
    from fp8_b200 import ops

    x = _gen((16, 128, 32, 32), seed=31)
    ops.quantize_current(x)  # warm-up outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        q, s = ops.quantize_current(x)
    x.copy_(_gen((16, 128, 32, 32), seed=32, scale=7.0))
    g.replay()
    torch.cuda.synchronize()
    q_ref, s_ref = oracle.quantize_current(x.cpu())
    assert np.float32(s.item()).tobytes() == s_ref.tobytes()
    assert np.array_equal(_bytes(q), q_ref)


@pytest.mark.parametrize("shapes", [
    ((128, 128, 32, 32), (128, 128, 3, 3)),   # config 2 input and weight
    ((2, 3, 4, 5), (7, 11)),                  # ragged tails in both
    ((1, 1, 1, 8192 * 3 + 5), (0,)),          # an empty tensor
])
def test_quantize_current_pair_matches_two_calls(cuda, shapes):
    from fp8_b200 import ops

    x = _gen(shapes[0], seed=41, scale=3.0)
    w = _gen(shapes[1], seed=42, scale=0.05) if shapes[1] != (0,) else torch.empty(0, dtype=torch.bfloat16, device=cuda)
    xq, sx, wq, sw = ops.quantize_current_pair(x, w)
    for q, s, t in ((xq, sx, x), (wq, sw, w)):
        q_ref, s_ref = oracle.quantize_current(t.cpu())
        assert np.float32(s.item()).tobytes() == s_ref.tobytes()
        assert np.array_equal(_bytes(q), q_ref)


def test_quantize_current_pair_unaligned_falls_back(cuda):
    from fp8_b200 import ops

    base = _gen((1, 1, 1, 4099), seed=43)
    x = base[..., 1:]
    w = _gen((64, 64, 3, 3), seed=44, scale=0.05)
    xq, sx, wq, sw = ops.quantize_current_pair(x, w)
    for q, s, t in ((xq, sx, x), (wq, sw, w)):
        q_ref, s_ref = oracle.quantize_current(t.cpu())
        assert np.float32(s.item()).tobytes() == s_ref.tobytes()
        assert np.array_equal(_bytes(q), q_ref)


def test_quantize_delayed_scale_fold_over_the_counter_ring(cuda):
    """The current scale is folded by the last CTA of the cast launch, on a ticket counter that each launch
    takes from a ring and leaves at zero.  More launches than the ring holds, with grids from 1 CTA to many
    (ragged sizes and the scalar path included): every scale equals amax / 448 of its own tensor."""
    from fp8_b200 import ops

    sizes = [8, 13, 4096, 65536 + 5, 1 << 20, 3 * (1 << 21)]
    xs = [_gen((n,), seed=100 + i, scale=0.5 + i) for i, n in enumerate(sizes)]
    xs.append(_gen((4097,), seed=99, scale=3.0)[1:])  # 2 bytes off alignment: the scalar kernel
    xs.append(torch.zeros(4096, dtype=torch.bfloat16, device=cuda))  # amax 0: scale 1
    amax = [np.float32(x.float().abs().max().item()) for x in xs]
    expect = torch.tensor([a / np.float32(448.0) if a > 0 else np.float32(1.0) for a in amax], device=cuda)
    prev = torch.tensor(0.01, dtype=torch.float32, device=cuda)
    got = []
    for i in range(8192 + 64):
        _, s = ops.quantize_delayed(xs[i % len(xs)], prev)
        got.append(s)
    got = torch.stack(got).view(-1, 1)
    torch.cuda.synchronize()
    n = len(xs)
    for k in range(n):
        assert torch.equal(got[k::n].view(-1), expect[k].expand(got[k::n].numel())), k
    assert ops.device_error() == 0


def test_quantize_delayed_window_replayed_in_cuda_graph(cuda):
    """The fold inside a captured graph: each replay writes the new scale at the history position and steps it."""
    from fp8_b200 import ops

    x = _gen((16, 128, 32, 32), seed=41)
    win = torch.zeros(8, dtype=torch.float32, device=cuda)
    win[0] = 0.02
    pos = torch.zeros((), dtype=torch.int64, device=cuda)
    ops.quantize_delayed_window(x, win, pos, True)  # warm-up outside capture: pos -> 1
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        q, used = ops.quantize_delayed_window(x, win, pos, True)
    scales = []
    for r in range(3):
        x.copy_(_gen((16, 128, 32, 32), seed=42 + r, scale=1.0 + r))
        prev_max = win.max().item()
        g.replay()
        torch.cuda.synchronize()
        q_ref, s_ref = oracle.quantize_delayed(x.cpu(), np.float32(prev_max))
        assert np.array_equal(_bytes(q), q_ref)
        assert used.item() == np.float32(prev_max)
        scales.append(s_ref)
        assert pos.item() == 2 + r
        assert win[1 + r].item() == float(s_ref)


@pytest.mark.parametrize("shape", [(128, 128, 32, 32), (128, 256, 16, 16), (1, 8, 1024, 1024), (32, 128, 32, 32)])
def test_resident_quantize_matches_two_pass_and_oracle(cuda, shape):
    """The one-launch shared-memory-resident current quantize (tensors of >= 6 MB whose
    per-SM shares fit in shared memory) gives the two-pass kernels' and the oracle's bytes
    and scales, alone and paired with a weight, eagerly and replayed from a CUDA graph."""
    from fp8_b200 import _lib, ops

    g = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(*shape, generator=g) * 3.0).to(torch.bfloat16).contiguous(memory_format=torch.channels_last)
    w = (torch.randn(128, 128, 3, 3, generator=g) * 0.05).to(torch.bfloat16).contiguous(
        memory_format=torch.channels_last)
    xd, wd = x.to(cuda), w.to(cuda)
    qr, sr = oracle.quantize_tensor(x)
    qwr, swr = oracle.quantize_tensor(w)
    try:
        results = {}
        for resident in (True, False):
            _lib.set_quantize_resident(resident)
            q, s = ops.quantize_current(xd)
            xq, sx, wq, sw = ops.quantize_current_pair(xd, wd)
            results[resident] = (q, s, xq, sx, wq, sw)
        _lib.set_quantize_resident(True)
        if shape == (128, 128, 32, 32):  # config 2's conv input and weight fit one resident launch together
            n0 = _lib.kernel_launch_count()
            ops.quantize_current_pair(xd, wd)
            torch.cuda.synchronize()
            assert _lib.kernel_launch_count() - n0 == 1
        # captured and replayed
        static = xd.clone()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            ops.quantize_current(static)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            gq, gs = ops.quantize_current(static)
        static.copy_(xd * 2)
        graph.replay()
        torch.cuda.synchronize()
        q2r, s2r = oracle.quantize_tensor((x.float() * 2).to(torch.bfloat16).contiguous(
            memory_format=torch.channels_last))
    finally:
        _lib.set_quantize_resident(True)
    for q, s, xq, sx, wq, sw in results.values():
        assert torch.equal(q.cpu().view(torch.uint8), qr.view(torch.uint8)) and s.item() == sr.item()
        assert torch.equal(xq.cpu().view(torch.uint8), qr.view(torch.uint8)) and sx.item() == sr.item()
        assert torch.equal(wq.cpu().view(torch.uint8), qwr.view(torch.uint8)) and sw.item() == swr.item()
    assert torch.equal(gq.cpu().view(torch.uint8), q2r.view(torch.uint8)) and gs.item() == s2r.item()
    assert _lib.device_error() == 0


@pytest.mark.parametrize("kind", ["finite", "nan", "inf"])
def test_resident_quantize_special_values(cuda, kind):
    """The resident launch's three casts against the oracle at config 2's size: every finite
    bf16 value with |x| <= 1024 and -0 in the tensor (no NaN: the cast without the clamp),
    the same with NaN planted in several CTAs' slices (amax ignores NaN; the clamped cast),
    and with +-inf (amax inf: the double-reciprocal cast); alone and paired with a weight."""
    from fp8_b200 import _lib, ops

    shape = (128, 128, 32, 32)
    n = int(np.prod(shape))
    g = torch.Generator().manual_seed(7)
    flat = (torch.randn(n, generator=g) * 3.0).to(torch.bfloat16).view(torch.int16).numpy().copy()
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    vals = oracle.bf16_bits_to_f32(bits)
    finite = bits[np.isfinite(vals) & (np.abs(vals) <= 1024.0)]
    flat[12345:12345 + finite.size] = finite.view(np.int16)
    flat[n - finite.size:] = finite[::-1].view(np.int16)
    flat[[1, n // 2, n - finite.size - 2]] = np.int16(-32768)  # -0
    if kind == "nan":
        flat[[0, n // 3, 2 * n // 3 + 5, n - 1]] = np.array([0x7FC0, 0xFFC0, 0x7F81, 0xFFFF],
                                                            dtype=np.uint16).view(np.int16)
    if kind == "inf":
        flat[[777, n // 2 + 1]] = np.array([0x7F80, 0xFF80], dtype=np.uint16).view(np.int16)
    x = torch.from_numpy(flat).view(torch.bfloat16).reshape(shape)
    w = (torch.randn(128, 128, 3, 3, generator=g) * 0.05).to(torch.bfloat16)
    qr, sr = oracle.quantize_current(x)
    qwr, swr = oracle.quantize_current(w)
    xd, wd = x.to(cuda), w.to(cuda)
    _lib.set_quantize_resident(True)
    n0 = _lib.kernel_launch_count()
    q, s = ops.quantize_current(xd)
    xq, sx, wq, sw = ops.quantize_current_pair(xd, wd)
    torch.cuda.synchronize()
    assert _lib.kernel_launch_count() - n0 == 2  # one resident launch each
    for got, gs, ref, rs in ((q, s, qr, sr), (xq, sx, qr, sr), (wq, sw, qwr, swr)):
        assert np.float32(gs.item()).tobytes() == np.float32(rs).tobytes(), (kind, gs.item(), rs)
        b = _bytes(got)
        bad = np.nonzero(b != ref)[0]
        assert bad.size == 0, f"{kind}: {bad.size} mismatches at {bad[:5]}: {b[bad[:5]]} vs {ref[bad[:5]]}"
    assert _lib.device_error() == 0
