"""DDPM UNet training step on B200: CUDA-graph captured, data parallel over NCCL.

What one step does (the reference's captured step, train.py:104-149 with the
loss of ddpm.py:174-215):

    x_t = sqrt(abar_t) x + sqrt(1 - abar_t) eps     t ~ U{0..T-1}, eps ~ N(0, 1)
    loss = mse(UNet(x_t, t), eps)                    bf16 autocast, FP8 convs
    backward -> (data parallel) bf16 gradient all-reduce -> clip_grad_norm(1.0)
    -> fused AdamW -> EMA of the weights (beta 0.9999)

Data parallelism: every rank holds a full replica and its own batch.  The
gradients are averaged with NCCL all-reduces of bf16 buckets (4 MB), each
launched on a side stream as soon as backward has produced every gradient of
the bucket (post-accumulate-grad hooks), so the exchange overlaps the rest of
backward; the step joins the side stream before clipping.  FP8 scales and the
delayed-scaling windows stay rank-local (the reference has no distributed code;
this is the data-parallel step of BASELINE config 5).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.distributed as dist
import torch.nn.functional as F

from .optim import FusedAdamWEMA
from .unet import UNet, UNetConfig


# ----------------------------------------------------------------------------- diffusion
class LinearSchedule:
    """Linear beta schedule of ddpm.py:122-131 (betas 1e-4 .. 0.02 over T steps, computed in fp64)."""

    def __init__(self, max_t: int = 1000, device: torch.device | str = "cuda"):
        scale = max_t / 1000
        betas = torch.linspace(1e-4 / scale, 0.02 / scale, max_t, dtype=torch.float64)
        self.alpha_bars = torch.cumprod(1.0 - betas, dim=0).float().to(device)
        self.max_t = max_t

    def mix(self, x: torch.Tensor, eps: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        """x_t = sqrt(abar_t) x + sqrt(1 - abar_t) eps (ddpm.py:199-202)."""
        ab = self.alpha_bars[t][:, None, None, None]
        return ab.sqrt() * x + (1.0 - ab).sqrt() * eps

    def noise(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(x_t, eps, t) for a batch (ddpm.py:190-206)."""
        t = torch.randint(0, self.max_t, (x.shape[0],), device=x.device)
        eps = torch.randn_like(x)
        return self.mix(x, eps, t), eps, t


def diffusion_loss(model: torch.nn.Module, x: torch.Tensor, sched: LinearSchedule) -> torch.Tensor:
    x_t, eps, t = sched.noise(x)
    return F.mse_loss(model(x_t, t), eps)


# ----------------------------------------------------------------------------- gradient all-reduce
class BucketedAllReduce:
    """Average gradients across ranks in bf16 buckets, overlapped with backward.

    Buckets first follow the reverse parameter order; the first backward records
    the order in which gradients actually become ready, and the buckets are then
    rebuilt in that order (as DDP does), so a bucket does not wait for a gradient
    that backward produces last (e.g. the time-embedding weights, whose gradients
    come from one GEMM at the very end).  For each bucket a hook counts the
    gradients that have been accumulated; the last one launches, on
    ``comm_stream``, the pack to a flat bf16 buffer (one cat), the all-reduce
    (NCCL averages in the collective; other backends sum, then scale), and the
    unpack into the fp32 gradients (one multi-tensor copy).  ``finish()`` makes
    the current stream wait for the side stream.
    """

    def __init__(self, params: list[torch.nn.Parameter], group=None, bucket_bytes: int = 25 << 20):
        self.group = group
        self.world = dist.get_world_size(group)
        self.params = [p for p in params if p.requires_grad]
        self.bucket_bytes = bucket_bytes
        # CPU tensors (gloo, host-side tests) reduce synchronously, without a side stream.
        self.comm_stream = torch.cuda.Stream(self.params[0].device) if self.params[0].is_cuda else None
        self.avg_in_collective = dist.get_backend(group) == "nccl"
        self._build(list(reversed(self.params)))
        self.order: list[torch.nn.Parameter] | None = []  # readiness order of the first backward
        self.handles = [p.register_post_accumulate_grad_hook(self._on_grad) for p in self.params]
        self.launched = 0

    def _build(self, ordered: list[torch.nn.Parameter]) -> None:
        self.buckets: list[list[torch.nn.Parameter]] = []
        cur, size = [], 0
        for p in ordered:
            cur.append(p)
            size += p.numel() * 2
            if size >= self.bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self.flat = [torch.empty(sum(p.numel() for p in b), device=b[0].device, dtype=torch.bfloat16)
                     for b in self.buckets]
        self.pending = [len(b) for b in self.buckets]
        self.bucket_of = {}
        for i, b in enumerate(self.buckets):
            for p in b:
                self.bucket_of[p] = i
        # per-bucket views of the flat buffer, one per gradient (for the multi-tensor unpack)
        self.views = []
        for b, flat in zip(self.buckets, self.flat):
            off, vs = 0, []
            for p in b:
                vs.append(flat[off:off + p.numel()].view(p.shape))
                off += p.numel()
            self.views.append(vs)

    def bytes_per_step(self) -> int:
        return sum(f.numel() * 2 for f in self.flat)

    def start(self) -> None:
        self.pending = [len(b) for b in self.buckets]
        self.launched = 0

    def _on_grad(self, p: torch.nn.Parameter) -> None:
        if self.order is not None:
            self.order.append(p)
        i = self.bucket_of[p]
        self.pending[i] -= 1
        if self.pending[i] == 0:
            self._launch(i)

    def _reduce(self, i: int) -> None:
        bucket, flat = self.buckets[i], self.flat[i]
        torch.cat([p.grad.reshape(-1) for p in bucket], out=flat)  # fp32 -> bf16 pack
        if self.avg_in_collective:
            dist.all_reduce(flat, op=dist.ReduceOp.AVG, group=self.group)
        else:
            dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group)
            flat.div_(self.world)
        torch._foreach_copy_([p.grad for p in bucket], self.views[i])  # bf16 -> fp32 unpack

    def _launch(self, i: int) -> None:
        if self.comm_stream is None:
            self._reduce(i)
        else:
            self.comm_stream.wait_stream(torch.cuda.current_stream(self.flat[i].device))
            with torch.cuda.stream(self.comm_stream):
                self._reduce(i)
        self.launched += 1

    def finish(self) -> None:
        if self.launched != len(self.buckets):
            raise RuntimeError(f"only {self.launched} of {len(self.buckets)} gradient buckets were reduced")
        if self.comm_stream is not None:
            torch.cuda.current_stream(self.flat[0].device).wait_stream(self.comm_stream)
        if self.order is not None:
            order, self.order = self.order, None
            index = {p: i for i, p in enumerate(self.params)}
            ids = [index[p] for p in order] if len(order) == len(self.params) and len(set(order)) == len(order) \
                else []
            box = [ids]
            dist.broadcast_object_list(box, src=dist.get_global_rank(self.group, 0) if self.group else 0,
                                       group=self.group)  # every rank buckets in rank 0's order
            if box[0]:
                if self.comm_stream is not None:
                    torch.cuda.current_stream(self.flat[0].device).synchronize()  # old buffers are idle
                self._build([self.params[i] for i in box[0]])

    def remove(self) -> None:
        for h in self.handles:
            h.remove()


# ----------------------------------------------------------------------------- the step
@dataclass
class TrainConfig:
    batch_size: int = 128
    lr: float = 2e-4
    max_t: int = 1000
    ema_beta: float = 0.9999
    grad_clip: float = 1.0
    warmup_iters: int = 3
    allreduce_bucket_mb: float = 4.0  # bf16 gradient bucket size of the data-parallel all-reduce (4 MB: 18.25 ms vs 18.47 ms at 25 MB, 2 x B200)
    # clip + AdamW + EMA of the parameters in one pass (fp8_b200.optim); torch's AdamW otherwise
    fused_optimizer: bool = True


class EMA:
    """Exponential moving average of the floating-point state (ddpm.py:10-25)."""

    def __init__(self, model: torch.nn.Module, beta: float):
        self.beta = beta
        self.src = [v for v in model.state_dict().values() if v.is_floating_point()]
        self.avg = [v.detach().clone() for v in self.src]

    @torch.no_grad()
    def update(self) -> None:
        torch._foreach_mul_(self.avg, self.beta)
        torch._foreach_add_(self.avg, self.src, alpha=1.0 - self.beta)


class GraphedTrainStep:
    """The captured training step; ``step(images)`` copies the batch in and replays."""

    def __init__(self, model: UNet, cfg: TrainConfig, device: torch.device, dp_group=None, use_graph: bool = True,
                 external_noise: bool = False):
        self.model = model
        self.cfg = cfg
        self.device = device
        self.sched = LinearSchedule(cfg.max_t, device)
        self.params = [p for p in model.parameters() if p.requires_grad]
        self.ema = EMA(model, cfg.ema_beta)
        if cfg.fused_optimizer:
            avg_of = {v.data_ptr(): a for v, a in zip(self.ema.src, self.ema.avg)}
            self.opt = FusedAdamWEMA(self.params, lr=cfg.lr, max_grad_norm=cfg.grad_clip,
                                     ema=[avg_of[p.data_ptr()] for p in self.params], ema_beta=cfg.ema_beta)
            ptrs = {p.data_ptr() for p in self.params}
            # the floating-point buffers (scale histories) keep the foreach EMA
            self.ema_rest = [(v, a) for v, a in zip(self.ema.src, self.ema.avg) if v.data_ptr() not in ptrs]
        else:
            self.opt = torch.optim.AdamW(self.params, lr=cfg.lr, fused=True, capturable=True)
        self.dp = BucketedAllReduce(self.params, dp_group, int(cfg.allreduce_bucket_mb * (1 << 20))) \
            if dist.is_initialized() and \
            dist.get_world_size(dp_group) > 1 else None
        if self.dp is not None and model.parameters().__next__().is_cuda:
            # The one-launch variants (weight-gradient conversion, current quantize) are cooperative
            # launches that need every SM; next to NCCL kernels on the comm stream they would wait for
            # the all-reduce to drain instead of overlapping it, so data parallel uses the two-launch forms.
            from . import _lib
            _lib.set_wgrad_fused(False)
            _lib.set_quantize_resident(False)
        cin, res = model.config.in_channels, model.config.in_resolution
        self.static_batch = torch.zeros(cfg.batch_size, cin, res, res, device=device).to(
            memory_format=torch.channels_last)
        # external_noise: the step takes its timesteps and noise from these buffers (step(images, t, eps))
        # instead of drawing them, so that runs of different models see the same draws
        self.external_noise = external_noise
        self.static_t = torch.zeros(cfg.batch_size, dtype=torch.int64, device=device)
        self.static_eps = torch.zeros_like(self.static_batch)
        self.loss_acc = torch.zeros((), device=device)
        self.graph = None
        self.use_graph = use_graph

    def _body(self) -> torch.Tensor:
        # Gradients are dropped, not zeroed: backward then hands each parameter its
        # gradient tensor instead of adding it into a zeroed one (one kernel fewer
        # per parameter).  Under graph capture those tensors come from the graph's
        # pool and keep their addresses on every replay.
        self.opt.zero_grad(set_to_none=True)
        if self.dp is not None:
            self.dp.start()
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16):
            if self.external_noise:
                x_t = self.sched.mix(self.static_batch, self.static_eps, self.static_t)
                loss = F.mse_loss(self.model(x_t, self.static_t), self.static_eps)
            else:
                loss = diffusion_loss(self.model, self.static_batch, self.sched)
        self.loss_acc.add_(loss.detach())
        loss.backward()
        if self.dp is not None:
            self.dp.finish()
        if self.cfg.fused_optimizer:
            self.opt.step()  # clip, AdamW and the parameters' EMA
            if self.ema_rest:
                with torch.no_grad():
                    avg = [a for _, a in self.ema_rest]
                    torch._foreach_mul_(avg, self.cfg.ema_beta)
                    torch._foreach_add_(avg, [v for v, _ in self.ema_rest], alpha=1.0 - self.cfg.ema_beta)
        else:
            torch.nn.utils.clip_grad_norm_(self.params, max_norm=self.cfg.grad_clip)
            self.opt.step()
            self.ema.update()
        return loss

    def prepare(self) -> None:
        """Eager warm-up iterations on a side stream (they also fill the delayed-scaling
        windows, train.py:114-128), then capture."""
        self.model.train()
        if dist.is_available() and dist.is_initialized():
            # every rank built the same model: give each rank its own dropout masks
            with torch.no_grad():
                for m in self.model.modules():
                    seed = getattr(m, "dropout_seed", None)
                    if isinstance(seed, torch.Tensor):
                        seed.add_(dist.get_rank() << 40)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(self.cfg.warmup_iters):
                self._body()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        if self.use_graph:
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self._body()
        self.loss_acc.zero_()

    def step(self, images: torch.Tensor | None = None, t: torch.Tensor | None = None,
             eps: torch.Tensor | None = None) -> None:
        if images is not None:
            self.static_batch.copy_(images, non_blocking=True)
        if t is not None:
            self.static_t.copy_(t, non_blocking=True)
        if eps is not None:
            self.static_eps.copy_(eps, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._body()

    def release(self) -> None:
        """Drop the graph (before tearing the process group down) and the hooks."""
        self.graph = None
        if self.dp is not None:
            self.dp.remove()


def build_model(fp8: bool = True, scaling: str = "delayed", attn_resolutions=(16,), p_drop: float = 0.1,
                device: torch.device | str = "cuda", seed: int = 0, fused_norm: bool = True,
                fused_resample: bool | None = None, plain: bool = False, skip_empty: bool = False,
                fp8_attention: bool = False, extended_shapes: bool = False) -> UNet:
    """The reference UNet; ``fused_norm`` / ``fused_resample`` (default: as ``fused_norm``) route its
    norm -> activation chains and its resampling + concatenation to this library's kernels.
    ``plain``: the reference's op structure throughout (every FP8 conv a ``triton_conv2d_fp8`` call,
    scale windows kept by torch ops in the module).  ``skip_empty``: ``fp8_history_skip_empty``.
    ``fp8_attention``: the attention blocks on the FP8 attention kernels.  ``extended_shapes``:
    ``fp8_extended_shapes`` (FP8 also for the 3x3 convs outside the reference's whitelist)."""
    torch.manual_seed(seed)
    if plain:
        fused_norm, fused_resample = False, False
    fr = fused_norm if fused_resample is None else fused_resample
    cfg = UNetConfig(fp8_convs_enabled=fp8, fp8_scaling_type=scaling, attn_resolutions=list(attn_resolutions),
                     p_drop=p_drop, fused_norm=fused_norm, fused_resample=fr, fused_residual=fr,
                     batched_time_embed=fr, fused_skip_cast=fr, batched_weight_cast=fr,
                     device_scale_history=not plain, fp8_history_skip_empty=skip_empty,
                     fp8_attention=fp8_attention, fp8_extended_shapes=extended_shapes)
    model = UNet(cfg).to(memory_format=torch.channels_last)
    return model.to(device)


def images_per_second(batch: int, world: int, ms_per_step: float) -> float:
    return batch * world / (ms_per_step * 1e-3)


__all__ = ["LinearSchedule", "diffusion_loss", "BucketedAllReduce", "TrainConfig", "EMA", "GraphedTrainStep",
           "build_model", "images_per_second", "math"]
