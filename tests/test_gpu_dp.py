"""Data-parallel UNet training step on two GPUs (NCCL, one process per GPU):
after CUDA-graph steps on different data the replicas' parameters stay
bit-identical (the bucketed bf16 all-reduce averages the same gradients into
every rank) and have moved from the initial weights.  Skipped on one GPU."""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results) -> None:
    import torch.distributed as dist

    from fp8_b200.train import GraphedTrainStep, TrainConfig, build_model

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        model = build_model(fp8=True, scaling="delayed", device=dev, seed=0)
        init = torch.cat([p.detach().float().flatten() for p in model.parameters()]).sum().item()
        step = GraphedTrainStep(model, TrainConfig(batch_size=16), dev)
        step.prepare()
        g = torch.Generator().manual_seed(50 + rank)
        for _ in range(3):
            step.step((torch.rand(16, 3, 32, 32, generator=g) * 2 - 1).to(dev))
        torch.cuda.synchronize()
        flat = torch.cat([p.detach().float().flatten() for p in model.parameters()])
        digest = torch.stack([flat.sum().double(), flat.abs().sum().double(), (flat * flat).sum().double()])
        gathered = [torch.empty_like(digest) for _ in range(world)]
        dist.all_gather(gathered, digest)
        results[rank] = (init, [t.tolist() for t in gathered], bool(step.loss_acc.isfinite().item()))
        step.release()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_dp_step_keeps_replicas_identical():
    world = 2
    manager = mp.Manager()
    results = manager.dict()
    mp.spawn(_worker, args=(world, _free_port(), results), nprocs=world, join=True)
    init0, digests0, finite0 = results[0]
    _, digests1, finite1 = results[1]
    assert finite0 and finite1
    assert digests0 == digests1                 # both ranks saw the same all-gathered digests
    assert digests0[0] == digests0[1]           # and the replicas are bit-identical
    assert digests0[0][0] != init0              # training moved the weights
