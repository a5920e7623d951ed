"""GPU pin of the B200 UNet path against the reference's own unet.py / ddpm.py.

``tests/golden/unet_reference.npz`` was made by running the reference's
``diffusion/unet.py`` and ``diffusion/ddpm.py`` unchanged (FP8 convs through the
CPU oracle, everything else in fp32; tests/golden/make_unet_golden.py) on
seeded weights and inputs.  Here the same weights and inputs run on the B200
under bf16 autocast, as the reference's train.py runs them, in two forms:

* ``plain``: the reference's op structure; every FP8 conv is a call of
  ``fp8_b200.fp8_kernels.triton_conv2d_fp8`` exactly as unet.py:62-94 makes it
  (scale windows updated by torch ops in the module);
* ``fused``: the production path (fused norm -> e4m3 kernels, device-side
  scale histories, batched weight quantize, fused resampling / residual joins).

Both must reproduce the reference's output, loss, parameter gradients and, for
delayed scaling, every FP8 conv's scale windows after three passes: weight
scales bit for bit (they depend on the weights alone), activation and dY
scales within bf16-autocast noise, including the scale 1.0 that the
reference's first, uncalibrated pass leaves in the dY windows of the
``conv_1`` convs.

A last test runs the plain model the way the reference's train.py does
(train.py:104-149, 250-253): ``torch.compile`` on the model, three warm-up
iterations on a side stream, fwd + bwd + clip + fused AdamW captured in one
CUDA graph and replayed, and compares it step by step with eager execution.
"""

from __future__ import annotations

import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"

# Tolerances.  The B200 path computes the non-FP8 layers in bf16 (autocast), so
# the inputs of its FP8 convs differ from the fp32 reference run's by bf16
# rounding and some e4m3 bytes land one step apart; through 44 FP8 convs these
# flips add up to the same distance that separates the reference's own FP8 run
# from its fp32 run on the same inputs (FP8 rounding noise, measured from the
# fixture itself).  Outputs and gradients must stay within 1.5x that noise
# floor; the loss within 1 %; activation and dY scales within the same floor;
# weight scales, the 1.0 sentinels and window positions exactly.
NOISE_FACTOR = 1.5
LOSS_RTOL = 1e-2
UNCALIBRATED_RTOL = 5e-2  # first delayed pass: FP8 convs output 0, the rest is bf16 vs fp32


def _gen():
    spec = importlib.util.spec_from_file_location("make_unet_golden", GOLDEN_DIR / "make_unet_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def fx():
    return dict(np.load(GOLDEN_DIR / "unet_reference.npz"))


def _config(fp8: bool, scaling: str, plain: bool):
    from fp8_b200.unet import UNetConfig

    kw = dict(_gen().MODEL_KW, fp8_convs_enabled=fp8, fp8_scaling_type=scaling)
    if plain:
        kw.update(fused_norm=False, fused_resample=False, device_scale_history=False, fused_residual=False,
                  batched_time_embed=False, fused_skip_cast=False, batched_weight_cast=False)
    return UNetConfig(**kw)


def _model(cuda, fp8: bool, scaling: str, plain: bool):
    from fp8_b200.unet import UNet

    torch.manual_seed(0)
    model = UNet(_config(fp8, scaling, plain)).to(memory_format=torch.channels_last)
    _gen().seeded_parameters(model)
    return model.to(cuda).train()


def _pass(model, fx, tag: str, s: int, cuda):
    xt = torch.from_numpy(fx[f"{tag}_xt_{s}"]).to(cuda).contiguous(memory_format=torch.channels_last)
    t = torch.from_numpy(fx[f"{tag}_t_{s}"]).to(cuda)
    eps = torch.from_numpy(fx[f"{tag}_eps_{s}"]).to(cuda)
    model.zero_grad(set_to_none=True)
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
        y = model(xt, t)
        loss = F.mse_loss(y, eps)
    loss.backward()
    torch.cuda.synchronize()
    return y.detach().float().cpu(), loss.item()


def _rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    return ((a - b).norm() / b.norm()).item()


def _grad_errors(model, ref: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    probe = _gen().grad_probe(model)
    scale = np.maximum(ref[:, 0], 1e-3 * ref[:, 0].max())
    return np.abs(probe[:, 0] - ref[:, 0]) / scale, np.abs(probe[:, 1] - ref[:, 1]) / scale


def _fp8_noise(fx) -> tuple[float, float, float]:
    """How far the reference's FP8 run (current scaling) is from its fp32 run on the same
    inputs: output rel L2 and the 95th percentiles of the per-parameter gradient errors."""
    out = _rel_l2(torch.from_numpy(fx["cur_out"][0]), torch.from_numpy(fx["fp32_out"][0]))
    ref = fx["fp32_grad_probe"]
    scale = np.maximum(ref[:, 0], 1e-3 * ref[:, 0].max())
    cur = fx["cur_grad_probe"]
    return (out, float(np.percentile(np.abs(cur[:, 0] - ref[:, 0]) / scale, 95)),
            float(np.percentile(np.abs(cur[:, 1] - ref[:, 1]) / scale, 95)))


def _check_pass(y, loss, fx, tag: str, s: int, what: str, out_tol: float) -> float:
    ref_y = torch.from_numpy(fx[f"{tag}_out"][s])
    err = _rel_l2(y, ref_y)
    ref_loss = float(fx[f"{tag}_loss"][s])
    print(f"{what} pass {s}: output rel L2 {err:.4f} (bound {out_tol:.4f}), loss {loss:.5f} vs {ref_loss:.5f}")
    assert err <= out_tol, (what, s, err)
    assert abs(loss - ref_loss) <= LOSS_RTOL * ref_loss, (what, s, loss, ref_loss)
    return err


def _check_grads(model, fx, tag: str, what: str) -> None:
    _, n95, p95 = _fp8_noise(fx)
    en, ep = _grad_errors(model, fx[f"{tag}_grad_probe"])
    print(f"{what} gradients: norm err median {np.median(en):.4f} p95 {np.percentile(en, 95):.4f} "
          f"(reference FP8 vs fp32 p95 {n95:.4f}); probe p95 {np.percentile(ep, 95):.4f} (reference {p95:.4f})")
    assert np.percentile(en, 95) <= NOISE_FACTOR * n95 + 0.02, (what, np.sort(en)[-10:])
    assert np.percentile(ep, 95) <= NOISE_FACTOR * p95 + 0.02, (what, np.sort(ep)[-10:])


def test_fp32_unet_on_gpu_matches_reference(cuda, fx):
    """FP8 off, fp32 without autocast (TF32 off): the torch-op path on the B200 computes
    what the reference's unet.py computes, to fp32 accumulation order."""
    prev = torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32
    torch.backends.cudnn.allow_tf32 = torch.backends.cuda.matmul.allow_tf32 = False
    try:
        model = _model(cuda, False, "current", plain=True)
        xt = torch.from_numpy(fx["fp32_xt_0"]).to(cuda).contiguous(memory_format=torch.channels_last)
        t = torch.from_numpy(fx["fp32_t_0"]).to(cuda)
        eps = torch.from_numpy(fx["fp32_eps_0"]).to(cuda)
        y = model(xt, t)
        loss = F.mse_loss(y, eps)
        loss.backward()
        err = _rel_l2(y.detach().cpu(), torch.from_numpy(fx["fp32_out"][0]))
        assert err <= 1e-4, err
        assert abs(loss.item() - float(fx["fp32_loss"][0])) <= 1e-5 * float(fx["fp32_loss"][0])
        en, ep = _grad_errors(model, fx["fp32_grad_probe"])
        assert en.max() <= 1e-3 and ep.max() <= 1e-3, (en.max(), ep.max())
    finally:
        torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("plain", [True, False], ids=["plain", "fused"])
def test_current_scaling_unet_matches_reference(cuda, fx, plain):
    model = _model(cuda, True, "current", plain)
    y, loss = _pass(model, fx, "cur", 0, cuda)
    what = "plain" if plain else "fused"
    _check_pass(y, loss, fx, "cur", 0, what, NOISE_FACTOR * _fp8_noise(fx)[0])
    _check_grads(model, fx, "cur", what)


@pytest.mark.parametrize("plain", [True, False], ids=["plain", "fused"])
def test_delayed_scaling_unet_matches_reference(cuda, fx, plain):
    from fp8_b200.unet import Conv2dFP8

    model = _model(cuda, True, "delayed", plain)
    what = "plain" if plain else "fused"
    for s in range(len(fx["del_loss"])):
        y, loss = _pass(model, fx, "del", s, cuda)
        tol = UNCALIBRATED_RTOL if s == 0 else NOISE_FACTOR * _fp8_noise(fx)[0]
        _check_pass(y, loss, fx, "del", s, what, tol)
    _check_grads(model, fx, "del", what)

    mods = dict(model.named_modules())
    names = list(fx["del_window_names"])
    assert sorted(names) == sorted(n for n, m in mods.items() if isinstance(m, Conv2dFP8))
    ref = fx["del_windows"]
    slots = ref.shape[2]
    sentinels = 0
    # an activation / dY scale is one extreme element of its tensor: it carries the FP8 noise floor
    scale_rtol = NOISE_FACTOR * _fp8_noise(fx)[0]
    for name, rw in zip(names, ref):
        m = mods[name]
        acts = m.amax_window_acts[:slots].cpu().numpy()
        wts = m.amax_window_weights[:slots].cpu().numpy()
        dys = m.amax_window_dy[:slots].cpu().numpy()
        assert int(m.window_pos.item()) == int(rw[3][0]), name
        np.testing.assert_array_equal(wts, rw[1], err_msg=f"{what} {name} weight scales")
        np.testing.assert_allclose(acts, rw[0], rtol=scale_rtol, atol=0, err_msg=f"{what} {name} input scales")
        one = rw[2] == 1.0
        sentinels += int(one.sum())
        np.testing.assert_array_equal(dys[one], rw[2][one], err_msg=f"{what} {name} dY sentinel")
        np.testing.assert_allclose(dys[~one], rw[2][~one], rtol=scale_rtol, atol=0, err_msg=f"{what} {name} dY scales")
    assert sentinels > 0  # the reference's uncalibrated first pass leaves dY scale 1.0 behind


def test_drop_in_under_torch_compile_and_cuda_graph(cuda, fx):
    """train.py:104-149 with the drop-in ops: compiled model, side-stream warm-up,
    captured fwd + bwd + clip + fused AdamW, replays; step by step against eager."""
    steps, warm = 3, 3
    inputs = []
    g = torch.Generator().manual_seed(9)
    for _ in range(warm + steps):
        xt = (torch.randn(2, 3, 32, 32, generator=g)).to(cuda).contiguous(memory_format=torch.channels_last)
        t = torch.randint(0, 1000, (2,), generator=g).to(cuda)
        eps = torch.randn(2, 3, 32, 32, generator=g).to(cuda)
        inputs.append((xt, t, eps))

    def make():
        model = _model(cuda, True, "delayed", plain=True)
        opt = torch.optim.AdamW(model.parameters(), lr=1e-4, fused=True, capturable=True)
        return model, opt

    def body(model, opt, static):
        opt.zero_grad(set_to_none=True)
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            loss = F.mse_loss(model(static[0], static[1]), static[2])
        loss.backward()
        torch.nn.utils.clip_grad_norm_(model.parameters(), max_norm=1.0)
        opt.step()
        return loss.detach()

    # eager
    model_e, opt_e = make()
    eager = [body(model_e, opt_e, inp).item() for inp in inputs]

    # compiled + graphed
    model_c, opt_c = make()
    compiled = torch.compile(model_c)
    static = tuple(x.clone() for x in inputs[0])
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graphed = []
    with torch.cuda.stream(side):
        for i in range(warm):
            for dst, src in zip(static, inputs[i]):
                dst.copy_(src)
            graphed.append(body(compiled, opt_c, static).item())
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    opt_c.zero_grad(set_to_none=True)
    with torch.cuda.graph(graph):
        loss_static = body(compiled, opt_c, static)
    for i in range(warm, warm + steps):
        for dst, src in zip(static, inputs[i]):
            dst.copy_(src)
        graph.replay()
        graphed.append(loss_static.item())
    torch.cuda.synchronize()
    del graph

    print("eager", eager, "compiled+graphed", graphed)
    for i, (a, b) in enumerate(zip(graphed, eager)):
        assert np.isfinite(a) and abs(a - b) <= 2e-2 * abs(b), (i, a, b)
    advanced = 0
    for (na, a), (nb, b) in zip(model_c.named_buffers(), model_e.named_buffers()):
        if na.endswith("window_pos"):  # FP8 convs step once per pass; the others never run FP8
            assert int(a.item()) == int(b.item()) and int(b.item()) in (0, warm + steps), na
            advanced += int(b.item()) == warm + steps
    assert advanced >= 40
