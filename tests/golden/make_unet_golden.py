"""Golden fixtures of the reference UNet and DDPM loss, run by the reference's own code.

Runs in the development container only (needs the reference checkout):

    python tests/golden/make_unet_golden.py /path/to/reference

It imports the reference package (``diffusion/unet.py``, ``diffusion/ddpm.py``)
unchanged.  Its FP8 convs go through ``oracle/ref_fp8_kernels_cpu.py``, a CPU
restatement of the reference's ``triton_conv2d_fp8`` installed under the name
``diffusion.fp8_kernels`` before the package is imported (unet.py:10 imports
only ``SUPPORTED_UNET_SHAPES`` and ``triton_conv2d_fp8`` from it).  The model
runs in fp32 on the CPU, with ``torch.compile`` disabled (``forward_batch`` is
decorated with it, ddpm.py:208).

Model: BASELINE config 4's architecture (base 128, mults (1,2,2,2), 2 residual
blocks, GroupNorm(32), attention at 16x16 and the middle stage) with dropout 0
so the results are deterministic, batch 2, every parameter overwritten by
``seeded_parameters`` (values drawn per parameter name, so any model with the
same state-dict names gets the same weights).  Recorded, as ``unet_reference.npz``:

* the linear schedule's alpha_bars (ddpm.py:122-131) and one noised batch of
  ``DiffusionWrapper.noise_batch`` (x0, t, eps, x_t; ddpm.py:190-206);
* ``fp32``: FP8 off.  UNet output, ``forward_batch`` loss (ddpm.py:208-215) and,
  per parameter, the gradient's L2 norm and its dot product with a seeded
  random direction (``grad_probe``);
* ``cur``: FP8 convs with current scaling, the same quantities;
* ``del``: FP8 convs with delayed scaling over three forward+backward passes on
  three batches (no weight update), each pass's output and loss, the gradient
  probes of the last pass, and every FP8 conv's scale windows (first 4 slots)
  and window position afterwards (unet.py:69-91, fp8_kernels.py:841-889).
"""

from __future__ import annotations

import os
import sys
import zlib
from pathlib import Path

os.environ["TORCHDYNAMO_DISABLE"] = "1"  # run forward_batch (ddpm.py:208) eagerly

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
OUT = HERE / "unet_reference.npz"
BATCH = 2
MODEL_KW = dict(in_channels=3, base_hidden=128, scales=[1, 2, 2, 2], n_heads=4, p_drop=0.0, attn_resolutions=[16],
                in_resolution=32, n_resblocks=2)
DELAYED_STEPS = 3
WINDOW_SLOTS = 4


def seeded_parameters(model: torch.nn.Module, seed: int = 11) -> None:
    """Overwrite every parameter with values drawn from a generator seeded by its name:
    matrices and conv kernels with std fan_in**-0.5, 1-D weights 1 + 0.1 N(0, 1), biases 0.1 N(0, 1).
    (Replaces the reference's zero inits of conv_2, attention out and the output conv,
    unet.py:145-146, 178-179, 355-357, so that every path carries signal.)"""
    with torch.no_grad():
        for name, p in model.named_parameters():
            g = torch.Generator().manual_seed(seed * 1_000_003 + zlib.crc32(name.encode()))
            if p.ndim >= 2:
                v = torch.randn(p.shape, generator=g) * p[0].numel() ** -0.5
            elif name.endswith("weight"):
                v = 1.0 + 0.1 * torch.randn(p.shape, generator=g)
            else:
                v = 0.1 * torch.randn(p.shape, generator=g)
            p.copy_(v.to(p.dtype))


def grad_probe(model: torch.nn.Module) -> np.ndarray:
    """Per parameter (in sorted name order): [||grad||_2, <grad, r>] with r a seeded
    N(0, 1) direction of the parameter's shape (0, 0 for a missing gradient)."""
    rows = []
    for name, p in sorted(model.named_parameters(), key=lambda kv: kv[0]):
        g = p.grad
        if g is None:
            rows.append((0.0, 0.0))
            continue
        g = g.detach().float().cpu()
        r = torch.randn(p.shape, generator=torch.Generator().manual_seed(zlib.crc32(name.encode()) + 7))
        rows.append((g.norm().item(), (g * r).sum().item()))
    return np.asarray(rows, dtype=np.float64)


def batch_inputs(seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return torch.rand(BATCH, 3, 32, 32, generator=g) * 2 - 1


def _import_reference(reference_root: str):
    sys.path.insert(0, str(HERE.parent.parent / "oracle"))
    import ref_fp8_kernels_cpu

    sys.modules["diffusion.fp8_kernels"] = ref_fp8_kernels_cpu
    sys.path.insert(0, reference_root)
    from diffusion.ddpm import DiffusionWrapper  # the reference modules, unchanged
    from diffusion.unet import UNet, UNetConfig

    return UNet, UNetConfig, DiffusionWrapper


def _run(UNet, UNetConfig, DiffusionWrapper, fp8: bool, scaling: str, steps: int, out: dict, tag: str) -> None:
    torch.manual_seed(0)
    model = UNet(UNetConfig(**MODEL_KW, fp8_convs_enabled=fp8, fp8_scaling_type=scaling))
    model = model.to(memory_format=torch.channels_last)
    seeded_parameters(model)
    model.train()
    ddpm = DiffusionWrapper(model, schedule_type="linear", max_t=1000, in_dim=32, device="cpu")
    record = {}
    noise = ddpm.noise_batch

    def noise_rec(x, t=None):
        res = noise(x, t)
        record["noised"] = res
        return res

    ddpm.noise_batch = noise_rec
    model.register_forward_hook(lambda mod, args, y: record.__setitem__("out", y))
    outs, losses = [], []
    for step in range(steps):
        model.zero_grad(set_to_none=True)
        x0 = batch_inputs(100 + step).to(memory_format=torch.channels_last)
        torch.manual_seed(1000 + step)
        loss = ddpm.forward_batch(x0)  # noise_batch -> model -> mse (ddpm.py:208-215)
        x_t, _, eps, t = record["noised"]
        loss.backward()
        outs.append(record["out"].detach().float().numpy())
        losses.append(loss.item())
        out[f"{tag}_x0_{step}"] = x0.numpy()
        out[f"{tag}_eps_{step}"] = eps.numpy()
        out[f"{tag}_t_{step}"] = t.numpy()
        out[f"{tag}_xt_{step}"] = x_t.detach().numpy()
    out[f"{tag}_out"] = np.stack(outs)
    out[f"{tag}_loss"] = np.asarray(losses)
    out[f"{tag}_grad_probe"] = grad_probe(model)
    if fp8 and scaling == "delayed":
        names, win = [], []
        for name, m in model.named_modules():
            if hasattr(m, "amax_window_acts"):
                names.append(name)
                win.append(np.stack([m.amax_window_acts[:WINDOW_SLOTS].numpy(),
                                     m.amax_window_weights[:WINDOW_SLOTS].numpy(),
                                     m.amax_window_dy[:WINDOW_SLOTS].numpy(),
                                     np.full(WINDOW_SLOTS, float(m.window_pos.item()), dtype=np.float32)]))
        out[f"{tag}_window_names"] = np.asarray(names)
        out[f"{tag}_windows"] = np.stack(win)
    if tag == "fp32":
        out["alpha_bars"] = ddpm.alpha_bars.numpy()
        out["param_names"] = np.asarray(sorted(n for n, _ in model.named_parameters()))


def main(reference_root: str) -> None:
    UNet, UNetConfig, DiffusionWrapper = _import_reference(reference_root)
    out: dict[str, np.ndarray] = {}
    _run(UNet, UNetConfig, DiffusionWrapper, False, "current", 1, out, "fp32")
    _run(UNet, UNetConfig, DiffusionWrapper, True, "current", 1, out, "cur")
    _run(UNet, UNetConfig, DiffusionWrapper, True, "delayed", DELAYED_STEPS, out, "del")
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {Path(__file__).name} <checkout of the reference repository>")
    main(sys.argv[1])
