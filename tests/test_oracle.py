"""CPU tests: pin the oracle against torch's e4m3 cast and the reference kernels' golden outputs."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fp8_oracle as oracle


def _torch_e4m3(v: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()


def test_encoder_matches_torch_on_every_bf16_value():
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    v = oracle.bf16_bits_to_f32(bits)
    v = v[np.isfinite(v)]
    for s in [1.0, 0.5, 3.0, 1 / 448.0, 0.0123, 1e-3, 17.7, 2.0**-20, 2.0**20]:
        with np.errstate(over="ignore"):
            t = np.fmax(np.float32(-448), np.fmin(v / np.float32(s), np.float32(448)))
        assert np.array_equal(oracle.e4m3_encode(t), _torch_e4m3(t)), s


def test_double_reciprocal_multiply_equals_fp32_division():
    """The GPU cast computes x / s as RN32(RN64(x * RN64(1 / s))).  Check that this
    equals IEEE fp32 division for every finite bf16 x and many fp32 scales with full
    24-bit significands (the CPU restatement of the argument in quantize.cuh)."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    v = oracle.bf16_bits_to_f32(bits)
    v = v[np.isfinite(v)]
    rng = np.random.default_rng(1234)
    scales = (rng.random(300) * 2.0 ** rng.integers(-40, 40, 300)).astype(np.float32)
    scales = np.concatenate([scales, np.float32([1.0, 0.1, 1 / 3, 448.0, 1 / 448, 2.0**-126, 3.4e38])])
    v64 = v.astype(np.float64)
    with np.errstate(over="ignore", under="ignore"):
        for s in scales:
            r = np.float64(1.0) / np.float64(s)
            assert np.array_equal((v64 * r).astype(np.float32), v / s), s


def test_encoder_ties_round_to_even():
    allb = np.arange(256, dtype=np.uint8)
    vals = torch.from_numpy(allb).view(torch.float8_e4m3fn).float().numpy()
    fin = np.unique(vals[np.isfinite(vals)])
    mids = ((fin[1:].astype(np.float64) + fin[:-1]) / 2).astype(np.float32)
    assert np.array_equal(oracle.e4m3_encode(mids), _torch_e4m3(mids))
    # and one fp32 ulp either side of every midpoint
    up = np.nextafter(mids, np.float32(np.inf))
    dn = np.nextafter(mids, np.float32(-np.inf))
    assert np.array_equal(oracle.e4m3_encode(up), _torch_e4m3(up))
    assert np.array_equal(oracle.e4m3_encode(dn), _torch_e4m3(dn))


def test_decoder_roundtrip():
    allb = np.arange(256, dtype=np.uint8)
    d = oracle.e4m3_decode(allb)
    ref = torch.from_numpy(allb).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(d), np.isnan(ref))
    assert np.array_equal(d[~np.isnan(d)], ref[~np.isnan(ref)])
    fin = ~np.isnan(d)
    assert np.array_equal(oracle.e4m3_encode(d[fin]), allb[fin])


def test_cast_clamp_semantics_follow_reference_min_max():
    # fp8_kernels.py:84-85 / :118-119: min(., 448) then max(-448, .), NaN-ignoring
    s = np.float32(0.0)  # uncalibrated delayed scale: x/0
    v = np.array([1.0, -1.0, 0.0, -0.0], dtype=np.float32)
    q = oracle.cast_with_scale(v, s)
    assert list(q) == [0x7E, 0xFE, 0x7E, 0x7E]  # +-inf -> +-448, 0/0 = NaN -> +448
    q = oracle.cast_with_scale(np.array([1000.0, -1000.0], dtype=np.float32), np.float32(1.0))
    assert list(q) == [0x7E, 0xFE]


def test_scale_of_zero_tensor_is_one():
    q, s = oracle.quantize_current(torch.zeros(2, 3, 4, 5, dtype=torch.bfloat16))
    assert s == np.float32(1.0) and not q.any()


def test_amax_ignores_nan():
    # fp8_kernels.py:62, :98: tl.max reduces with the GPU's max.f32, which returns the
    # other operand when one is NaN; only an all-NaN tensor falls back to scale 1.0
    v = np.array([1.5, np.nan, -7.0, 0.25], dtype=np.float32)
    assert oracle.amax_scale(v) == np.float32(np.float32(7.0) / np.float32(448.0))
    assert oracle.amax_scale(np.full(5, np.nan, dtype=np.float32)) == np.float32(1.0)
    q = oracle.cast_with_scale(v, oracle.amax_scale(v))
    assert q[1] == 0x7E and q[2] == 0xFE  # NaN -> +448 by the clamp; -amax -> -448


@pytest.mark.parametrize("name", ["randn", "zeros", "pow2", "ragged", "tiny"])
def test_quantize_scales_match_reference_kernels(golden, name):
    bits = golden[f"q_{name}_x"].reshape(-1)
    v = oracle.bf16_bits_to_f32(bits)
    assert oracle.amax_scale(v).tobytes() == golden[f"q_{name}_scale"].tobytes()
    # delayed: the reported scale is the tensor's own one
    q, s_curr = oracle.quantize_delayed(
        torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16), float(golden[f"q_{name}_delayed_prev"][0])
    )
    assert s_curr.tobytes() == golden[f"q_{name}_delayed_scale"].tobytes()


CONV_CASES = ["c128x8", "c256x4", "c128to256x16", "c128x32"]


def _conv_case(golden, tag):
    b, cin, cout, h, w = (int(v) for v in golden[f"{tag}_dims"])

    def fp8(arr, shape_nhwc):
        t = torch.from_numpy(arr.reshape(shape_nhwc)).view(torch.float8_e4m3fn)
        return t.permute(0, 3, 1, 2)  # logical NCHW view of NHWC bytes (channels_last)

    def bf16(arr, shape_nhwc):
        return torch.from_numpy(arr.reshape(shape_nhwc).view(np.int16)).view(torch.bfloat16).permute(0, 3, 1, 2)

    sx, sw, sdy = (float(v) for v in golden[f"{tag}_scales"])
    return dict(
        dims=(b, cin, cout, h, w),
        xq=fp8(golden[f"{tag}_xq"], (b, h, w, cin)),
        wq=fp8(golden[f"{tag}_wq"], (cout, 3, 3, cin)),
        dyq=fp8(golden[f"{tag}_dyq"], (b, h, w, cout)),
        sx=sx, sw=sw, sdy=sdy,
        y=bf16(golden[f"{tag}_y"], (b, h, w, cout)),
        dx=bf16(golden[f"{tag}_dx"], (b, h, w, cin)),
        dw=bf16(golden[f"{tag}_dw"], (cout, 3, 3, cin)),
        dyt=golden[f"{tag}_dyt"],
    )


@pytest.mark.parametrize("tag", CONV_CASES)
def test_conv_oracle_matches_reference_kernels(golden, tag):
    c = _conv_case(golden, tag)
    y = oracle.conv_fwd(c["xq"], c["wq"], c["sx"], c["sw"])
    dx = oracle.conv_dx(c["dyq"], c["wq"], c["sdy"], c["sw"])
    dw = oracle.conv_dw(c["xq"], c["dyq"], c["sx"], c["sdy"])
    # same fp32 products, different summation order: at most a bf16 rounding step apart
    assert oracle.max_rel_err(y, c["y"]) < 1e-2
    assert oracle.max_rel_err(dx, c["dx"]) < 1e-2
    assert oracle.max_rel_err(dw, c["dw"]) < 1e-2
    # The interpreter's bf16 stores truncate; with the same truncation the oracle's
    # fp32 results reproduce the reference bits except where summation order
    # moves a value across a bf16 boundary.
    rz = oracle.round_bf16_toward_zero
    for f32, ref in (
        (oracle.conv_fwd(c["xq"], c["wq"], c["sx"], c["sw"], f32=True), c["y"]),
        (oracle.conv_dx(c["dyq"], c["wq"], c["sdy"], c["sw"], f32=True), c["dx"]),
        (oracle.conv_dw(c["xq"], c["dyq"], c["sx"], c["sdy"], f32=True), c["dw"]),
    ):
        same = (rz(f32).float() == ref.float()).float().mean().item()
        assert same > 0.999, same


@pytest.mark.parametrize("tag", CONV_CASES)
def test_golden_quantized_inputs_are_oracle_casts(golden, tag):
    # the fixture inputs were quantised with the oracle: re-derive and compare
    c = _conv_case(golden, tag)
    b, cin, cout, h, w = c["dims"]
    dyt = c["dyt"]
    nhwc = golden[f"{tag}_dyq"].reshape(b * h * w, cout)
    assert np.array_equal(dyt, nhwc.T)  # reference transpose_fp8_2d_kernel semantics


def test_attention_oracle_close_to_exact_attention():
    """The FP8 attention restatement stays within e4m3 noise of exact fp32 attention
    (forward and backward), and its per-head scales are the reference quantize's."""
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(2, 64, 768, generator=g).to(torch.bfloat16)
    o, lse, sc = oracle.attention_fwd(qkv, 4)
    ex = oracle.attention_exact(qkv, 4)
    assert ((o.float() - ex).norm() / ex.norm()).item() < 0.1
    heads = qkv.float().view(2, 64, 3, 4, 64)
    for b in range(2):
        for h in range(4):
            for t in range(3):
                _, s_ref = oracle.quantize_tensor(heads[b, :, t, h, :].to(torch.bfloat16).contiguous())
                assert sc[b, h, t].item() == s_ref.item()
    do = (torch.randn(2, 64, 256, generator=g) * 0.01).to(torch.bfloat16)
    dqkv = oracle.attention_bwd(qkv, o, do, lse, 4)
    x = qkv.float().requires_grad_(True)
    xs = x.view(2, 64, 3, 4, 64).permute(2, 0, 3, 1, 4)
    oe = torch.nn.functional.scaled_dot_product_attention(xs[0], xs[1], xs[2]).transpose(1, 2).reshape(2, 64, 256)
    oe.backward(do.float())
    assert ((dqkv.float() - x.grad).norm() / x.grad.norm()).item() < 0.1
