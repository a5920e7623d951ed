"""CPU tests of the training-side host logic: the UNet's layout matches the
reference, its dispatch rule, and the data-parallel gradient all-reduce
(two gloo ranks in separate processes)."""

from __future__ import annotations

import json
import os
import socket
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fp8_b200.unet import Conv2dFP8, UNet, UNetConfig, fp8_conv_modules

FIXTURE = Path(__file__).resolve().parent / "golden" / "reference_unet_state_dict.json"


@pytest.mark.parametrize("name,attn", [("attn16", [16]), ("attn16_8", [16, 8])])
def test_state_dict_layout_matches_reference(name, attn):
    ref = json.loads(FIXTURE.read_text())[name]
    model = UNet(UNetConfig(attn_resolutions=attn, fp8_convs_enabled=True, fp8_scaling_type="delayed"))
    ours = [[k, list(v.shape), str(v.dtype)] for k, v in model.state_dict().items()]
    assert sorted(ours) == sorted(ref["state_dict"])
    assert sum(p.numel() for p in model.parameters()) == ref["params"]


def test_forward_shape_without_fp8_on_cpu():
    torch.manual_seed(0)
    model = UNet(UNetConfig(fp8_convs_enabled=False))
    x = torch.randn(2, 3, 32, 32)
    t = torch.randint(0, 1000, (2,))
    y = model(x, t)
    assert y.shape == x.shape
    assert torch.count_nonzero(y) == 0  # the output conv is zero-initialised (unet.py:355-357)


def test_swap_linears_replaces_the_unet_linears_and_keeps_the_state_dict():
    """The nn.Linear swap of the FP8 linear API: attention qkv / out projections, the blocks' time-embedding
    projections and the time MLP become FP8Linear sharing their parameters; the state_dict is unchanged."""
    from fp8_b200.linear import FP8Linear, swap_linears

    torch.manual_seed(0)
    model = UNet(UNetConfig(fp8_convs_enabled=True, fp8_scaling_type="delayed"))
    before = {k: v.data_ptr() for k, v in model.state_dict().items()}
    n_lin = sum(isinstance(m, torch.nn.Linear) for m in model.modules())
    assert swap_linears(model) == n_lin == 7 * 2 + 22 + 2
    assert all(isinstance(m, FP8Linear) for m in model.modules() if isinstance(m, torch.nn.Linear))
    after = {k: v.data_ptr() for k, v in model.state_dict().items()}
    assert after == before  # same keys, same tensors
    model2 = UNet(UNetConfig())
    assert swap_linears(model2, lambda name, lin: name in ("qkv", "out")) == 14


def test_fp8_dispatch_follows_whitelist():
    model = UNet(UNetConfig(fp8_convs_enabled=True))
    convs = fp8_conv_modules(model)
    assert len(convs) == 2 * (2 * 4 + 3 * 4 + 2)  # two convs per residual block
    c = Conv2dFP8(512, 256, fp8_convs_enabled=True)
    assert c.uses_fp8(torch.empty(1, 512, 16, 16))
    assert not c.uses_fp8(torch.empty(1, 512, 4, 4))  # 512->256 at 4x4 is not whitelisted
    assert not Conv2dFP8(128, 128, fp8_convs_enabled=False).uses_fp8(torch.empty(1, 128, 32, 32))
    with pytest.raises(ValueError):
        Conv2dFP8(128, 128, True, scaling_type="delayed")  # needs an amax history length


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_worker(rank: int, world: int, port: int, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fp8_b200.train import BucketedAllReduce

        torch.manual_seed(0)
        model = torch.nn.Sequential(torch.nn.Linear(16, 32), torch.nn.Tanh(), torch.nn.Linear(32, 8))
        data = [torch.randn(4, 16, generator=torch.Generator().manual_seed(100 + r)) for r in range(world)]
        # reference: the average of every rank's own gradient, computed locally
        ref = [torch.zeros_like(p) for p in model.parameters()]
        for r in range(world):
            model.zero_grad()
            model(data[r]).square().mean().backward()
            for acc, p in zip(ref, model.parameters()):
                acc += p.grad / world
        model.zero_grad()
        dp = BucketedAllReduce(list(model.parameters()), bucket_bytes=200)  # several buckets
        for _ in range(2):  # twice, to check that the per-step state resets
            model.zero_grad()
            dp.start()
            model(data[rank]).square().mean().backward()
            dp.finish()
        errs = [((p.grad - r).abs().max() / r.abs().max()).item() for p, r in zip(model.parameters(), ref)]
        results[rank] = (len(dp.buckets), max(errs))
        dp.remove()
    finally:
        dist.destroy_process_group()


def test_bucketed_allreduce_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_dp_worker, args=(2, _free_port(), results), nprocs=2, start_method="spawn")
        out = dict(results)
    assert set(out) == {0, 1}
    for n_buckets, err in out.values():
        assert n_buckets >= 2
        assert err < 1e-2  # bf16 all-reduce of fp32 gradients


def _dp_missing_worker(rank: int, world: int, port: int, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fp8_b200.train import BucketedAllReduce

        model = torch.nn.Linear(4, 4)
        dp = BucketedAllReduce(list(model.parameters()))
        dp.start()
        # no backward: finish() must refuse to continue with unreduced gradients
        try:
            dp.finish()
            results[rank] = "no error"
        except RuntimeError as e:
            results[rank] = str(e)
    finally:
        dist.destroy_process_group()


def test_bucketed_allreduce_detects_missing_gradients():
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        results = mgr.dict()
        mp.start_processes(_dp_missing_worker, args=(2, _free_port(), results), nprocs=2, start_method="spawn")
        out = dict(results)
    assert all("were reduced" in v for v in out.values()), out
