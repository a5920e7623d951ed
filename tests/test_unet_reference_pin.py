"""CPU pin of the re-implemented UNet and DDPM loss against the reference's own code.

``tests/golden/unet_reference.npz`` holds what the reference's ``diffusion/unet.py``
and ``diffusion/ddpm.py`` compute (tests/golden/make_unet_golden.py ran them,
unchanged, on seeded weights and inputs).  Here ``fp8_b200.unet.UNet`` with the
reference's op structure (no fused kernels, FP8 off) and ``fp8_b200.train``'s
schedule and noising run the same inputs on the CPU in fp32 and must give the
same numbers: the schedule exactly, the output, loss and every parameter
gradient to fp32 rounding.
"""

from __future__ import annotations

import importlib.util
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"


def _fixture_module():
    spec = importlib.util.spec_from_file_location("make_unet_golden", GOLDEN_DIR / "make_unet_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def fx():
    return dict(np.load(GOLDEN_DIR / "unet_reference.npz"))


def plain_config(fp8: bool, scaling: str = "current", **kw):
    """UNetConfig with the reference's op structure: every fused path off."""
    from fp8_b200.unet import UNetConfig

    gen = _fixture_module()
    base = dict(gen.MODEL_KW, fp8_convs_enabled=fp8, fp8_scaling_type=scaling, fused_norm=False,
                fused_resample=False, device_scale_history=False, fused_residual=False, batched_time_embed=False,
                fused_skip_cast=False, batched_weight_cast=False)
    base.update(kw)
    return UNetConfig(**base)


def test_schedule_and_noising_match_reference(fx):
    from fp8_b200.train import LinearSchedule

    sched = LinearSchedule(1000, "cpu")
    assert torch.equal(sched.alpha_bars, torch.from_numpy(fx["alpha_bars"]))
    for tag, steps in (("fp32", 1), ("cur", 1), ("del", 3)):
        for s in range(steps):
            x0 = torch.from_numpy(fx[f"{tag}_x0_{s}"])
            eps = torch.from_numpy(fx[f"{tag}_eps_{s}"])
            t = torch.from_numpy(fx[f"{tag}_t_{s}"])
            xt = sched.mix(x0, eps, t)
            torch.testing.assert_close(xt, torch.from_numpy(fx[f"{tag}_xt_{s}"]), rtol=1e-6, atol=1e-6)


def test_state_dict_names_match_reference(fx):
    from fp8_b200.unet import UNet

    model = UNet(plain_config(False))
    assert sorted(n for n, _ in model.named_parameters()) == list(fx["param_names"])


def test_fp32_unet_matches_reference_unet(fx):
    """FP8 off, fp32 on the CPU: output, DDPM loss and every gradient as the reference's."""
    from fp8_b200.unet import UNet

    gen = _fixture_module()
    torch.manual_seed(0)
    model = UNet(plain_config(False)).to(memory_format=torch.channels_last)
    gen.seeded_parameters(model)
    model.train()
    xt = torch.from_numpy(fx["fp32_xt_0"]).contiguous(memory_format=torch.channels_last)
    t = torch.from_numpy(fx["fp32_t_0"])
    eps = torch.from_numpy(fx["fp32_eps_0"])
    y = model(xt, t)
    loss = F.mse_loss(y, eps)
    loss.backward()

    ref_y = torch.from_numpy(fx["fp32_out"][0])
    assert (y.detach() - ref_y).abs().max().item() <= 1e-4 * ref_y.abs().max().item()
    assert abs(loss.item() - float(fx["fp32_loss"][0])) <= 1e-5 * float(fx["fp32_loss"][0])
    probe = gen.grad_probe(model)
    ref = fx["fp32_grad_probe"]
    assert probe.shape == ref.shape
    norm_ref = ref[:, 0]
    assert (norm_ref > 0).all()  # every parameter receives a gradient with these weights
    assert np.all(np.abs(probe[:, 0] - norm_ref) <= 1e-3 * norm_ref)
    assert np.all(np.abs(probe[:, 1] - ref[:, 1]) <= 1e-3 * norm_ref)
