"""GPU tests of the caller side: the delayed-scaling Conv2dFP8 module against a
CPU emulation of the reference semantics (unet.py:62-94, fp8_kernels.py:823-913),
the CUDA-graph training step, and the 200-step loss curve of the FP8 UNet
against the bf16 one (within 2 %)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import fp8_oracle as oracle

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _bf16_cl(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).contiguous(memory_format=torch.channels_last)


def test_delayed_conv_module_matches_reference_semantics(cuda):
    from fp8_b200.unet import Conv2dFP8

    torch.manual_seed(0)
    mod = Conv2dFP8(128, 128, fp8_convs_enabled=True, scaling_type="delayed", amax_history=8).to(cuda)
    mod = mod.to(memory_format=torch.channels_last)
    # a calibrated history (the reference fills it during warm-up iterations)
    with torch.no_grad():
        mod.amax_window_acts[3] = 0.011
        mod.amax_window_weights[5] = 0.0003
        mod.amax_window_dy[1] = 2e-5
    acts = mod.amax_window_acts.cpu().clone()
    wts = mod.amax_window_weights.cpu().clone()
    dys = mod.amax_window_dy.cpu().clone()
    pos = 0
    w = _bf16_cl(mod.conv.weight.detach()).cpu()
    g = torch.Generator().manual_seed(1)
    for step in range(3):
        x = _bf16_cl(torch.randn(4, 128, 32, 32, generator=g))
        dy = _bf16_cl(torch.randn(4, 128, 32, 32, generator=g) * 1e-2)
        xd = x.to(cuda).requires_grad_(True)
        y = mod(xd)
        y.backward(dy.to(cuda))

        # --- emulation of the reference (CPU oracle) ---
        x_hist, w_hist, dy_hist = acts.max(), wts.max(), dys.max()
        xq, x_curr = oracle.quantize_delayed(x, float(x_hist))
        wq, w_curr = oracle.quantize_delayed(w, float(w_hist))
        dyq, dy_curr = oracle.quantize_delayed(dy, float(dy_hist))
        xq_t, wq_t, dyq_t = oracle.bytes_like(xq, x), oracle.bytes_like(wq, w), oracle.bytes_like(dyq, dy)
        y_ref = oracle.conv_fwd(xq_t, wq_t, float(x_hist), float(w_hist))
        dx_ref = oracle.conv_dx(dyq_t, wq_t, float(dy_hist), float(w_hist))
        dw_ref = oracle.conv_dw(xq_t, dyq_t, float(x_hist), float(dy_hist))
        acts[pos] = float(x_curr)
        wts[pos] = float(w_curr)
        pos = (pos + 1) % 8
        dys[pos] = float(dy_curr)  # lands one slot after x / w (window_pos already advanced)

        assert oracle.max_rel_err(y, y_ref) <= TOL, step
        assert oracle.max_rel_err(xd.grad, dx_ref) <= TOL, step
        assert oracle.max_rel_err(mod.conv.weight.grad, dw_ref) <= TOL, step
        assert torch.equal(mod.amax_window_acts.cpu(), acts), step
        assert torch.equal(mod.amax_window_weights.cpu(), wts), step
        assert torch.equal(mod.amax_window_dy.cpu(), dys), step
        assert int(mod.window_pos.item()) == pos
        mod.conv.weight.grad = None


def test_uncalibrated_delayed_conv_is_finite_and_zero(cuda):
    """First call with all-zero windows: x/0 clamps to 448 and the output is acc * 0 (unet.py:49)."""
    from fp8_b200.unet import Conv2dFP8

    mod = Conv2dFP8(128, 256, fp8_convs_enabled=True, scaling_type="delayed", amax_history=4).to(cuda)
    x = _bf16_cl(torch.randn(2, 128, 32, 32)).to(cuda).requires_grad_(True)
    y = mod(x)
    y.backward(_bf16_cl(torch.randn(2, 256, 32, 32)).to(cuda))
    assert torch.isfinite(y).all() and torch.count_nonzero(y) == 0
    assert torch.isfinite(x.grad).all() and torch.count_nonzero(x.grad) == 0
    assert mod.amax_window_acts[0] > 0 and mod.amax_window_dy[1] > 0


def test_graphed_train_step_runs_and_updates(cuda):
    from fp8_b200.train import GraphedTrainStep, TrainConfig, build_model

    model = build_model(fp8=True, scaling="delayed", device=cuda)
    step = GraphedTrainStep(model, TrainConfig(batch_size=32), cuda)
    before = [p.detach().clone() for p in step.params]
    ema_before = [a.clone() for a in step.ema.avg]
    step.prepare()
    g = torch.Generator().manual_seed(0)
    for _ in range(5):
        step.step((torch.rand(32, 3, 32, 32, generator=g) * 2 - 1).to(cuda))
    torch.cuda.synchronize()
    loss = step.loss_acc.item() / 5
    assert np.isfinite(loss) and 0.05 < loss < 5.0
    assert any(not torch.equal(a, b) for a, b in zip(before, step.params))
    assert any(not torch.equal(a, b) for a, b in zip(ema_before, step.ema.avg))
    step.release()


LOSS_STEPS, LOSS_BATCH = 200, 128


def _loss_curve(cuda, **model_kw) -> np.ndarray:
    """200 CUDA-graph training steps (BASELINE config 4 architecture, synthetic uniform
    images).  Timesteps and noise come from one seeded host generator, so every model
    sees the same draws and the curves differ only by the models' arithmetic."""
    from fp8_b200.train import GraphedTrainStep, TrainConfig, build_model

    model = build_model(device=cuda, seed=0, **model_kw)
    step = GraphedTrainStep(model, TrainConfig(batch_size=LOSS_BATCH), cuda, external_noise=True)
    torch.manual_seed(1234)
    torch.cuda.manual_seed(1234)
    step.prepare()
    g = torch.Generator().manual_seed(7)
    data = [(torch.rand(LOSS_BATCH, 3, 32, 32, generator=g) * 2 - 1) for _ in range(8)]
    gn = torch.Generator().manual_seed(99)
    losses = []
    for i in range(LOSS_STEPS):
        t = torch.randint(0, 1000, (LOSS_BATCH,), generator=gn)
        eps = torch.randn(LOSS_BATCH, 3, 32, 32, generator=gn)
        step.step(data[i % len(data)].to(cuda), t.to(cuda), eps.to(cuda))
        losses.append(step.loss_acc.clone())
        step.loss_acc.zero_()
    torch.cuda.synchronize()
    step.release()
    return np.array([l.item() for l in losses])


def _curve_gap(curve: np.ndarray, ref: np.ndarray) -> tuple[float, float]:
    """(mean over steps 50-200 of |MA10(curve) - MA10(ref)| / MA10(ref),
        max over steps 50-200 of |MA50(curve) - MA50(ref)| / MA50(ref))."""
    def ma(c, k):
        return np.convolve(c, np.ones(k) / k, mode="valid")
    m10, r10 = ma(curve, 10)[41:], ma(ref, 10)[41:]  # windows ending at steps 50 .. 200
    m50, r50 = ma(curve, 50), ma(ref, 50)
    return float(np.mean(np.abs(m10 - r10) / r10)), float(np.max(np.abs(m50 - r50) / r50))


@pytest.fixture(scope="module")
def loss_curves(cuda):
    """The bf16 reference model (the reference's op structure, pinned to the reference's
    unet.py by tests/test_gpu_unet_reference.py) and the B200 FP8 paths."""
    return {
        "bf16": _loss_curve(cuda, fp8=False, plain=True),
        "fp8_current": _loss_curve(cuda, fp8=True, scaling="current"),
        "fp8_delayed_skip_empty": _loss_curve(cuda, fp8=True, scaling="delayed", skip_empty=True),
        "fp8_delayed_skip_empty_fp8_attention": _loss_curve(cuda, fp8=True, scaling="delayed", skip_empty=True,
                                                            fp8_attention=True),
        "fp8_delayed_skip_empty_extended": _loss_curve(cuda, fp8=True, scaling="delayed", skip_empty=True,
                                                       extended_shapes=True),
        "fp8_delayed": _loss_curve(cuda, fp8=True, scaling="delayed"),
        "fp8_delayed_plain": _loss_curve(cuda, fp8=True, scaling="delayed", plain=True),
    }


# Measured on a B200 (mean MA10 gap, max MA50 gap): FP8 current 0.13 %, 1.0 %; delayed with
# empty tensors recording 0 0.53 %, 1.8 %; the bf16 model with the fused norm kernels against
# the same model on torch ops 0.48 %, 1.1 %; delayed with the reference's history semantics
# 10.4 %, 16 % (fused) and 8.8 %, 16 % (the reference's op structure).
CURVE_MEAN_TOL = 0.02
CURVE_MA50_TOL = 0.03


@pytest.mark.parametrize("name", ["fp8_current", "fp8_delayed_skip_empty", "fp8_delayed_skip_empty_fp8_attention"])
def test_fp8_loss_curve_within_2pct_of_bf16(loss_curves, name):
    """North-star loss bar: over 200 steps the FP8 curve stays within 2 % of bf16 (mean of
    the 10-step moving average's relative gap over steps 50-200; the 50-step moving average
    within 3 % everywhere).  Both FP8 scalings meet it: current scaling (unet.py:24's default)
    and delayed scaling (train.py:230-231's fastest config) when an all-zero tensor records
    scale 0 in its history, also with the attention blocks on the FP8 attention kernels."""
    curve, ref = loss_curves[name], loss_curves["bf16"]
    assert np.isfinite(curve).all() and np.isfinite(ref).all()
    assert ref[-50:].mean() < 0.5 * ref[:10].mean()  # it trains
    mean_gap, ma50_gap = _curve_gap(curve, ref)
    print(f"{name}: mean MA10 gap {mean_gap:.4f}, max MA50 gap {ma50_gap:.4f}")
    assert mean_gap <= CURVE_MEAN_TOL, (name, mean_gap)
    assert ma50_gap <= CURVE_MA50_TOL, (name, ma50_gap)


def test_fp8_extended_shapes_loss_curve(loss_curves):
    """FP8 also for the 512 -> 256 conv at 4x4, which the reference's whitelist leaves in bf16
    (UNetConfig.fp8_extended_shapes, off by default).  Its mean MA10 gap stays within the 2 %
    bar (0.9 % measured), but its 50-step moving average has been measured up to 3.4 % from
    bf16 on one box (the split-K weight gradients add in a run-dependent order, so curves vary
    slightly between runs), above the 3 % excursion bound; that is why the option stays off."""
    curve, ref = loss_curves["fp8_delayed_skip_empty_extended"], loss_curves["bf16"]
    assert np.isfinite(curve).all() and curve[-50:].mean() < 0.5 * curve[:10].mean()
    mean_gap, ma50_gap = _curve_gap(curve, ref)
    print(f"fp8_delayed_skip_empty_extended: mean MA10 gap {mean_gap:.4f}, max MA50 gap {ma50_gap:.4f}")
    assert mean_gap <= CURVE_MEAN_TOL, mean_gap
    assert ma50_gap <= 0.05, ma50_gap


def test_delayed_gap_is_the_reference_history_semantics(loss_curves):
    """With the reference's delayed-scaling bookkeeping, the first (uncalibrated) pass leaves
    scale 1.0 (the scale of an all-zero tensor, finalize_amax_kernel) in the dY histories of
    every conv_1 and in the weight histories of the zero-initialised conv_2s; the history max
    keeps it for 1024 steps and e4m3 flushes those gradients / weights to zero.  The curve then
    trails bf16 by well over 2 % -- on the reference's own op structure (plain) as on the fused
    path -- and recording 0 for empty tensors removes the gap (test above)."""
    ref = loss_curves["bf16"]
    for name in ("fp8_delayed", "fp8_delayed_plain"):
        curve = loss_curves[name]
        assert np.isfinite(curve).all() and curve[-50:].mean() < 0.5 * curve[:10].mean()
        mean_gap, _ = _curve_gap(curve, ref)
        print(f"{name}: mean MA10 gap {mean_gap:.4f}")
        assert mean_gap > 0.04, (name, mean_gap)
    skip_gap, _ = _curve_gap(loss_curves["fp8_delayed_skip_empty"], ref)
    assert skip_gap < 0.5 * _curve_gap(loss_curves["fp8_delayed"], ref)[0]


def test_fused_norm_unet_as_accurate_as_torch_ops(cuda):
    """The fused GroupNorm/FiLM/SiLU path is as close to an fp32 UNet as the
    reference's torch-op bf16 path is (same weights, dropout off, bf16 convs to
    isolate the norm path): output and per-parameter gradient errors against
    fp32 no worse than 1.5x the torch-op path's."""
    from fp8_b200.train import build_model

    models = [build_model(fp8=False, device=cuda, seed=3, p_drop=0.0, fused_norm=f) for f in (True, False, False)]
    with torch.no_grad():
        for named in zip(*(m.named_parameters() for m in models)):
            a = named[0][1]
            if a.dim() == 4 and a.abs().max() == 0:  # zero-initialised conv_2 / output convs
                a.normal_(0, 0.02)
            for _, b in named[1:]:
                b.copy_(a)
    g = torch.Generator().manual_seed(11)
    x = (torch.rand(8, 3, 32, 32, generator=g) * 2 - 1).to(cuda).contiguous(memory_format=torch.channels_last)
    t = torch.randint(0, 1000, (8,), generator=g).to(cuda)
    outs, grads = [], []
    for i, m in enumerate(models):
        m.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=i < 2):
            y = m(x, t)
        y.float().square().mean().backward()
        outs.append(y.float())
        grads.append({n: p.grad.float() for n, p in m.named_parameters() if p.grad is not None})
    rel = lambda a, b: ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()  # noqa: E731
    fused_err, torch_err = rel(outs[0], outs[2]), rel(outs[1], outs[2])
    assert fused_err <= 1.5 * torch_err + 1e-3, (fused_err, torch_err)
    names = [n for n in grads[2] if grads[2][n].abs().max() > 0]
    g_fused = np.median([rel(grads[0][n], grads[2][n]) for n in names])
    g_torch = np.median([rel(grads[1][n], grads[2][n]) for n in names])
    assert g_fused <= 1.5 * g_torch + 1e-3, (g_fused, g_torch)


def test_batched_time_embedding_matches_per_block(cuda):
    """One GEMM for all blocks' time-embedding projections gives the UNet output and gradients of the
    per-block projections (max relative error <= 1e-2: the GEMMs' summation order may differ)."""
    from fp8_b200.train import build_model

    x = (torch.rand(4, 3, 32, 32) * 2 - 1).to(cuda).contiguous(memory_format=torch.channels_last)
    t = torch.randint(0, 1000, (4,)).to(cuda)
    res = []
    for batched in (True, False):
        m = build_model(fp8=False, device=cuda, seed=0, p_drop=0.0)
        m.config.batched_time_embed = batched
        with torch.no_grad():  # the zero-initialised branches would give zero gradients everywhere
            torch.manual_seed(1)
            for mod in m.modules():
                if isinstance(mod, torch.nn.Conv2d) and not mod.weight.any():
                    torch.nn.init.normal_(mod.weight, std=0.02)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = m(x, t)
        y.float().square().mean().backward()
        blk = m.down_stages[0].blocks[0]
        res.append((y.detach(), blk.t_embed_wb.mlp.weight.grad.clone(), m.time_embed[0].weight.grad.clone()))
    (ya, wa, ta), (yb, wb, tb) = res
    # the GEMMs may sum in another order: within bf16 rounding of the projections
    for u, v in ((ya, yb), (wa, wb), (ta, tb)):
        assert ((u - v).abs().max() / v.abs().max()).item() <= 1e-2


def test_fp8_extended_shapes_run_the_remaining_convs_in_fp8(cuda):
    """With fp8_extended_shapes the 512 -> 256 conv at 4x4 (outside SUPPORTED_UNET_SHAPES) runs in FP8 too;
    the step trains like the default configuration (loss within 2 % after a few steps)."""
    from fp8_b200.train import build_model
    from fp8_b200.unet import Conv2dFP8

    x = (torch.rand(8, 3, 32, 32) * 2 - 1).to(cuda).contiguous(memory_format=torch.channels_last)
    t = torch.randint(0, 1000, (8,)).to(cuda)
    losses = {}
    for ext in (False, True):
        m = build_model(fp8=True, scaling="delayed", device=cuda, seed=0, p_drop=0.0)
        m.config.fp8_extended_shapes = ext
        for mod in m.modules():
            if isinstance(mod, Conv2dFP8):
                mod.extended_shapes = ext
        opt = torch.optim.AdamW(m.parameters(), lr=2e-4)
        for _ in range(4):
            opt.zero_grad()
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = (m(x, t).float() - x).square().mean()
            loss.backward()
            opt.step()
        fp8_mods = [mod for mod in m.modules() if isinstance(mod, Conv2dFP8) and mod.window_pos.item() > 0]
        losses[ext] = (loss.item(), len(fp8_mods))
    assert losses[True][1] > losses[False][1]  # more convs took the FP8 path
    assert abs(losses[True][0] - losses[False][0]) <= 0.02 * abs(losses[False][0])


def test_unet_with_fp8_linears_trains_like_bf16_linears(cuda):
    """swap_linears puts the attention projections and the time-embedding MLP on the FP8 GEMM (the
    batched time-embedding GEMM is switched off so the blocks' projections run through their modules);
    a few AdamW steps give the loss of the bf16 linears within 2 %."""
    from fp8_b200.linear import FP8Linear, swap_linears
    from fp8_b200.train import build_model

    x = (torch.rand(8, 3, 32, 32) * 2 - 1).to(cuda).contiguous(memory_format=torch.channels_last)
    t = torch.randint(0, 1000, (8,)).to(cuda)
    losses = {}
    for fp8_lin in (False, True):
        m = build_model(fp8=True, scaling="delayed", device=cuda, seed=0, p_drop=0.0)
        m.config.batched_time_embed = False
        if fp8_lin:
            assert swap_linears(m) == 38
        opt = torch.optim.AdamW(m.parameters(), lr=2e-4)
        for _ in range(4):
            opt.zero_grad()
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = (m(x, t).float() - x).square().mean()
            loss.backward()
            opt.step()
        losses[fp8_lin] = loss.item()
        if fp8_lin:
            qkv = m.up_stages[2].attns[0].qkv
            assert isinstance(qkv, FP8Linear) and qkv.weight.grad is not None and qkv.weight.grad.abs().sum() > 0
    assert abs(losses[True] - losses[False]) <= 0.02 * abs(losses[False])


def test_empty_tensor_history_modes(cuda):
    """fp8_set_empty_tensor_history: an all-zero tensor records scale 1.0 in its history (mode
    0, the reference's finalize_amax_kernel value) or 0.0 (mode 1); a tensor with values records
    its scale either way, and the scale outputs keep the reference value."""
    from fp8_b200 import _lib, ops

    zeros = torch.zeros(2, 128, 8, 8, dtype=torch.bfloat16, device=cuda).contiguous(memory_format=torch.channels_last)
    vals = _bf16_cl(torch.randn(2, 128, 8, 8)).to(cuda)
    w_zero = torch.zeros(128, 128, 3, 3, device=cuda).contiguous(memory_format=torch.channels_last)
    w_vals = (torch.randn(128, 128, 3, 3) * 0.05).to(cuda).contiguous(memory_format=torch.channels_last)
    try:
        for mode, empty in ((0, 1.0), (1, 0.0)):
            _lib.set_empty_tensor_history(mode)
            win = torch.zeros(4, device=cuda)
            pos = torch.zeros((), dtype=torch.int64, device=cuda)
            ops.quantize_delayed_window(zeros, win, pos, True)
            ops.quantize_delayed_window(vals, win, pos, True)
            _, s_vals = oracle.quantize_tensor(vals.cpu())
            assert win[0].item() == empty and win[1].item() == float(s_vals.item()), mode
            assert int(pos.item()) == 2
            wins = [torch.zeros(4, device=cuda), torch.zeros(4, device=cuda)]
            poss = [torch.zeros((), dtype=torch.int64, device=cuda) for _ in range(2)]
            ops.quantize_weights_delayed([w_zero, w_vals], wins, poss)
            _, s_w = oracle.quantize_tensor(w_vals.to(torch.bfloat16).cpu())
            assert wins[0][0].item() == empty and wins[1][0].item() == float(s_w.item()), mode
            q, s = ops.quantize_delayed(zeros, torch.ones((), device=cuda))
            assert s.item() == 1.0  # the op's scale output is the reference's in both modes
    finally:
        _lib.set_empty_tensor_history(0)
