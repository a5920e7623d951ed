"""DDPM UNet with the reference's architecture, calling the B200 FP8 conv op.

This is the caller of the FP8 path (the reference's ``diffusion/unet.py``),
rebuilt here so that the training step can run on a machine without the
reference checkout.  Module and buffer names follow the reference one for one,
so ``state_dict``s are interchangeable:

* ``Conv2dFP8`` (unet.py:32-94): an ``nn.Conv2d`` 3x3 (``.conv``) plus, for
  delayed scaling, the windows ``amax_window_{weights,acts,dy}`` (they hold
  scales, amax/448) and ``window_pos``; shapes in ``SUPPORTED_UNET_SHAPES`` go to
  ``triton_conv2d_fp8``, everything else to the bf16 conv.
* ``ResidualBlock`` (unet.py:107-161), ``CHWAttention`` (:164-203), ``Stage``
  (:206-242), ``UNet`` (:245-388) with ``UNetConfig`` (:13-28).

Architecture (reference defaults used by BASELINE config 4: base 128, channel
multipliers (1, 2, 2, 2), 2 residual blocks per level, GroupNorm(32), SiLU,
dropout, attention at the listed resolutions plus the 4x4 middle stage, a
512-wide time-embedding MLP on a 128-wide sinusoidal embedding).
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, ops
from .attention import attention_supported, fp8_attention
from .delayed import ConvFP8Delayed, GroupNormActConvFP8Delayed, quantize_conv_weights
from .fp8_kernels import SUPPORTED_UNET_SHAPES, triton_conv2d_fp8
from .resample import downsample_nearest, residual_join, upsample_cat, upsample_cat_pair
from .weights import batch_cast_applies, cast_cat_weights_bf16, cast_weights_bf16
from .norm import GroupNormActConvFP8, fused_layer_norm_supported, fused_norm_supported, group_norm_act, layer_norm_bf16


@dataclass
class UNetConfig:
    in_channels: int = 3
    base_hidden: int = 128
    scales: list[int] = field(default_factory=lambda: [1, 2, 2, 2])
    n_heads: int = 4
    p_drop: float = 0.1
    attn_resolutions: list[int] = field(default_factory=lambda: [16])
    in_resolution: int = 32
    n_resblocks: int = 2
    fp8_convs_enabled: bool = False
    fp8_scaling_type: str = "current"
    fp8_amax_history: int = 1024
    # GroupNorm -> (FiLM) -> SiLU -> (dropout) chains as one fused CUDA op
    # (fp8_b200.norm) where the activation is a bf16 CUDA tensor; the reference's
    # separate torch ops otherwise.  No parameters or buffers depend on it.
    fused_norm: bool = True
    # nearest resampling + skip concatenation as single passes (fp8_b200.resample)
    fused_resample: bool = True
    # delayed scaling: the kernels read and update the scale histories on the
    # device (fp8_b200.delayed) instead of torch.max / scatter launches per conv;
    # the histories, scales and results are the same
    device_scale_history: bool = True
    # the residual joins (skip + h) / sqrt(2) as one pass (fp8_b200.resample.residual_join)
    fused_residual: bool = True
    # every block's time-embedding projection (all of them read the same embedding)
    # as one GEMM over the concatenated weights, instead of one small GEMM per block
    batched_time_embed: bool = True
    # FP8 also for the 3x3 convs outside SUPPORTED_UNET_SHAPES whose channel counts
    # the kernels take (multiples of 128; here the 512 -> 256 conv at 4x4), with
    # delayed scaling on device histories.  Off by default: the reference runs them
    # in bf16.
    fp8_extended_shapes: bool = False
    # an up stage's fp32 input (upsample + skip concatenation) and the bf16 copy autocast
    # makes of it for the first block's 1x1 skip conv, written by one pass; their two
    # gradients summed by the backward of that pass (needs fused_resample)
    fused_skip_cast: bool = True
    # the bf16 copies autocast makes of the bf16 layers' fp32 weights (attention projections,
    # 1x1 skip convs, time-embedding linears), and the casts of their gradients back, one
    # launch each way per step (fp8_b200.weights)
    batched_weight_cast: bool = True
    # delayed scaling: an all-zero tensor (conv_2's zero-initialised weight, or conv_1's output
    # gradient on the first, uncalibrated step) records scale 0 instead of the reference's 1.0 in
    # its history, so the history max is not held at 1.0 for the next fp8_amax_history steps
    # (fp8_b200._lib.set_empty_tensor_history).  Off by default: the reference records 1.0.
    # Needs device_scale_history.
    fp8_history_skip_empty: bool = False
    # the attention blocks' softmax(q k^T / sqrt(d)) v as the FP8 attention kernels
    # (fp8_b200.attention: e4m3 q, k, v per image and head, FP8 QK^T and PV) instead of the
    # reference's bf16 scaled_dot_product_attention (unet.py:197).  Off by default.
    fp8_attention: bool = False

    def as_dict(self):
        return asdict(self)


class Conv2dFP8(nn.Module):
    """3x3 / pad 1 conv; FP8 for whitelisted shapes, bf16 ``nn.Conv2d`` otherwise."""

    def __init__(self, in_channels: int, out_channels: int, fp8_convs_enabled: bool, scaling_type: str = "current",
                 amax_history: int | None = None, device_scale_history: bool = True, extended_shapes: bool = False):
        super().__init__()
        self.device_scale_history = device_scale_history
        self.extended_shapes = extended_shapes
        self._pre_weight = None  # (wq, sw) from a batched weight quantize, for the next forward
        self.used_fp8_delayed = False  # whether a forward since the UNet's last one ran the delayed FP8 path
        self.last_fp8_delayed = False  # whether the latest forward did (on device scale histories)
        self._dy_handoff = None  # (dy, e4m3 dy, scale) from the op that produced this conv's output gradient
        self._dx_add = None  # a second gradient of the normalised input, from the residual join
        self.last_fused_norm_input = None  # (data_ptr, shape, dtype) of x when forward_normed ran fused
        self.dgrad_relayout = False  # whether the data-grad of the last delayed FP8 forward re-lays the weights out
        if scaling_type not in ("current", "delayed"):
            raise ValueError(f"unknown FP8 scaling type {scaling_type!r}")
        self.conv = nn.Conv2d(in_channels, out_channels, (3, 3), stride=1, padding=1, bias=False)
        self.scaling_type = scaling_type
        self.fp8_convs_enabled = fp8_convs_enabled
        if scaling_type == "delayed":
            if amax_history is None:
                raise ValueError("delayed scaling needs amax_history")
            self.amax_history = amax_history
            # scale history (amax / 448) of the weights, inputs and output gradients
            self.register_buffer("amax_window_weights", torch.zeros(amax_history))
            self.register_buffer("amax_window_acts", torch.zeros(amax_history))
            self.register_buffer("amax_window_dy", torch.zeros(amax_history))
            self.register_buffer("window_pos", torch.zeros((), dtype=torch.long))

    def uses_fp8(self, x: torch.Tensor) -> bool:
        key = (x.shape[1], self.conv.weight.shape[0], x.shape[2], x.shape[3])
        if not self.fp8_convs_enabled:
            return False
        if key in SUPPORTED_UNET_SHAPES:
            return True
        return (self.extended_shapes and self.scaling_type == "delayed" and self.device_scale_history
                and key[0] % 128 == 0 and key[1] % 128 == 0)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        self.last_fp8_delayed = False
        if not self.uses_fp8(x):
            return self.conv(x)
        x = x.contiguous(memory_format=torch.channels_last)
        if self.scaling_type == "current":
            return triton_conv2d_fp8(x, self.conv.weight)
        if self.device_scale_history:
            pre, self._pre_weight = self._pre_weight, None
            self.used_fp8_delayed = self.last_fp8_delayed = True
            self.dgrad_relayout = ops.dgrad_needs_relayout(x.shape[0], x.shape[2], x.shape[3], x.shape[1],
                                                           self.conv.weight.shape[0])
            return ConvFP8Delayed.apply(x, self.conv.weight, self.amax_window_acts, self.amax_window_weights,
                                        self.amax_window_dy, self.window_pos, pre, self)
        with torch.no_grad():
            x_hist = torch.max(self.amax_window_acts)
            w_hist = torch.max(self.amax_window_weights)
        out, x_scale, w_scale = triton_conv2d_fp8(
            x, self.conv.weight, (x_hist, w_hist), (self.amax_window_dy, self.window_pos), do_delayed=True
        )
        with torch.no_grad():
            idx = self.window_pos.unsqueeze(0)
            self.amax_window_weights.scatter_(0, idx, w_scale.detach().unsqueeze(0))
            self.amax_window_acts.scatter_(0, idx, x_scale.detach().unsqueeze(0))
            self.window_pos.add_(1).remainder_(self.amax_history)
        return out


    def forward_normed(self, x: torch.Tensor, norm: nn.GroupNorm, film: torch.Tensor | None = None, p: float = 0.0,
                       seed: torch.Tensor | None = None, x_owner: "Conv2dFP8 | None" = None) -> torch.Tensor:
        """``self(group_norm_act(x, norm, film, p, seed))``.  With delayed scaling the
        group-norm pass writes this conv's e4m3 input itself (GroupNormActConvFP8).
        ``x_owner``: the delayed FP8 conv that produced x, whose backward then receives the
        e4m3 cast of x's gradient from the norm's backward."""
        self.last_fp8_delayed = False
        self.last_fused_norm_input = None
        if not (self.scaling_type == "delayed" and self.uses_fp8(x) and fused_norm_supported(x, norm)):
            return self(group_norm_act(x, norm, film, p, seed))
        if p > 0.0 and seed is None:
            raise ValueError("dropout needs a seed tensor")
        x = x.contiguous(memory_format=torch.channels_last)
        if self.device_scale_history:
            pre, self._pre_weight = self._pre_weight, None
            self.used_fp8_delayed = self.last_fp8_delayed = True
            self.last_fused_norm_input = (x.data_ptr(), x.shape, x.dtype)
            self.dgrad_relayout = ops.dgrad_needs_relayout(x.shape[0], x.shape[2], x.shape[3], x.shape[1],
                                                           self.conv.weight.shape[0])
            return GroupNormActConvFP8Delayed.apply(
                x, norm.weight, norm.bias, film, seed if p > 0.0 else None, self.conv.weight, self.amax_window_acts,
                self.amax_window_weights, self.amax_window_dy, self.window_pos, float(p), float(norm.eps),
                int(norm.num_groups), pre, self, x_owner)
        with torch.no_grad():
            x_hist = torch.max(self.amax_window_acts)
            w_hist = torch.max(self.amax_window_weights)
        out, x_scale, w_scale = GroupNormActConvFP8.apply(
            x, norm.weight, norm.bias, film, seed if p > 0.0 else None, self.conv.weight, x_hist, w_hist,
            self.amax_window_dy, self.window_pos, float(p), float(norm.eps), int(norm.num_groups))
        with torch.no_grad():
            idx = self.window_pos.unsqueeze(0)
            self.amax_window_weights.scatter_(0, idx, w_scale.unsqueeze(0))
            self.amax_window_acts.scatter_(0, idx, x_scale.unsqueeze(0))
            self.window_pos.add_(1).remainder_(self.amax_history)
        return out


class TimeEmbed(nn.Module):
    """Per-block projection of the time embedding to a (scale, shift) pair."""

    def __init__(self, embed_channels: int, channels: int):
        super().__init__()
        self.mlp = nn.Linear(embed_channels, channels, bias=False)

    def forward(self, t: torch.Tensor) -> torch.Tensor:
        return self.mlp(t)[:, :, None, None]


class ResidualBlock(nn.Module):
    def __init__(self, config: UNetConfig, in_chann: int, out_chann: int, p_drop: float = 0.0):
        super().__init__()
        conv = dict(fp8_convs_enabled=config.fp8_convs_enabled, scaling_type=config.fp8_scaling_type,
                    amax_history=config.fp8_amax_history, device_scale_history=config.device_scale_history,
                    extended_shapes=config.fp8_extended_shapes)
        self.conv_1 = Conv2dFP8(in_chann, out_chann, **conv)
        self.conv_2 = Conv2dFP8(out_chann, out_chann, **conv)
        self.norm1 = nn.GroupNorm(32, in_chann)
        self.norm2 = nn.GroupNorm(32, out_chann)
        self.t_embed_wb = TimeEmbed(4 * config.base_hidden, 2 * out_chann)
        self.skip_connection: nn.Module = (
            nn.Identity() if in_chann == out_chann else nn.Conv2d(in_chann, out_chann, (1, 1), bias=False)
        )
        self.dropout = nn.Dropout(p_drop)
        nn.init.zeros_(self.conv_2.conv.weight)
        self.fused_norm = config.fused_norm
        self.fused_residual = config.fused_residual
        self._emb = None  # this block's time-embedding projection, when the UNet computed it in a batch
        self._skip_in = None  # bf16 copy of the input for the 1x1 skip conv, when the UNet made one
        self._skip_w16 = None  # bf16 copy of the skip conv's weight, when the UNet made one
        self._seed = None  # this step's dropout seed, when the UNet drew all blocks' seeds at once
        # dropout mask seed of the fused path (device scalar, advanced every
        # training forward so a captured graph draws a new mask each replay)
        self.register_buffer("dropout_seed", torch.randint(0, 2**62, (), dtype=torch.int64), persistent=False)

    def _next_seed(self) -> torch.Tensor:
        seed = self.dropout_seed.clone()
        self.dropout_seed.add_(1)
        return seed

    def forward(self, x: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        emb, self._emb = self._emb, None  # set by the UNet's batched projection
        if emb is None:
            emb = self.t_embed_wb(t)
        if self.fused_norm and fused_norm_supported(x, self.norm1):
            h = self.conv_1.forward_normed(x, self.norm1)
            if fused_norm_supported(h, self.norm2) and emb.dtype == torch.bfloat16:
                p = self.dropout.p if self.training else 0.0
                seed, self._seed = self._seed, None
                if p > 0.0 and seed is None:
                    seed = self._next_seed()
                h = self.conv_2.forward_normed(h, self.norm2, emb, p, seed if p > 0.0 else None,
                                               x_owner=self.conv_1 if self.conv_1.last_fp8_delayed else None)
                return self._join(x, h)
        else:
            h = self.conv_1(F.silu(self.norm1(x)))
        scale, shift = torch.chunk(emb, chunks=2, dim=1)
        h = (scale + 1) * self.norm2(h) + shift
        h = self.conv_2(self.dropout(F.silu(h)))
        return self._join(x, h)

    def _join(self, x: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
        skip_in, self._skip_in = self._skip_in, None
        w16, self._skip_w16 = self._skip_w16, None
        src = x if skip_in is None else skip_in
        skip = self.skip_connection(src) if w16 is None else F.conv2d(src, w16, self.skip_connection.bias)
        if self.fused_residual:
            # h is conv_2's output: when that ran the delayed FP8 path, the join's backward also makes
            # the e4m3 cast of h's gradient for conv_2's backward.  With an identity skip whose x conv_1's
            # fused norm read as is, x's skip gradient is added inside that norm's backward.
            key = (x.data_ptr(), x.shape, x.dtype)
            skip_target = (self.conv_1 if isinstance(self.skip_connection, nn.Identity) and skip_in is None
                           and self.conv_1.last_fused_norm_input == key else None)
            return residual_join(skip, h, dy_target=self.conv_2 if self.conv_2.last_fp8_delayed else None,
                                 skip_target=skip_target)
        return (skip + h) / math.sqrt(2.0)


class CHWAttention(nn.Module):
    """Multi-head self-attention over the pixels of a [B, C, H, W] feature map."""

    def __init__(self, config: UNetConfig, hidden_size: int):
        super().__init__()
        self.fused_norm = config.fused_norm
        self.fused_residual = config.fused_residual
        self.fp8_attention = config.fp8_attention
        self.nh = config.n_heads
        self.qkv = nn.Linear(hidden_size, 3 * hidden_size, bias=False)
        self.out = nn.Linear(hidden_size, hidden_size, bias=False)
        self.norm = nn.LayerNorm(hidden_size)
        nn.init.zeros_(self.out.weight)
        self._w16 = None  # bf16 copies of (qkv, out) weights, when the UNet made them

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, c, h, w = x.shape
        tokens = x.flatten(2).transpose(1, 2)  # [B, HW, C]
        if self.fused_norm and tokens.is_contiguous() and fused_layer_norm_supported(tokens, self.norm):
            tokens = layer_norm_bf16(tokens, self.norm)  # bf16, what the qkv projection consumes
        else:
            tokens = self.norm(tokens)
        w16, self._w16 = self._w16, None
        qkv = self.qkv(tokens) if w16 is None else F.linear(tokens, w16[0], self.qkv.bias)
        if self.fp8_attention and attention_supported(qkv, self.nh):
            o = fp8_attention(qkv, self.nh)  # [B, HW, C], heads side by side as the out projection reads them
        else:
            q, k, v = qkv.chunk(3, dim=-1)
            heads = lambda z: z.unflatten(-1, (self.nh, c // self.nh)).transpose(1, 2)  # noqa: E731
            o = F.scaled_dot_product_attention(heads(q), heads(k), heads(v))
            o = o.transpose(1, 2).flatten(2)
        o = self.out(o) if w16 is None else F.linear(o, w16[1], self.out.bias)  # [B, HW, C]
        o = o.transpose(1, 2).reshape(b, c, h, w)
        if self.fused_residual:
            return residual_join(o, x)
        return (o + x) / math.sqrt(2.0)


class Stage(nn.Module):
    def __init__(self, config: UNetConfig, in_channels: int, hidden_channels: int, out_channels: int,
                 attention: bool = False, num_blocks: int = 2):
        super().__init__()
        self.num_blocks = num_blocks
        widths = [in_channels] + [hidden_channels] * (num_blocks - 1) + [out_channels]
        self.blocks = nn.ModuleList(
            ResidualBlock(config, widths[i], widths[i + 1], p_drop=config.p_drop) for i in range(num_blocks)
        )
        self.attns = nn.ModuleList(
            CHWAttention(config, widths[i + 1]) if attention else nn.Identity() for i in range(num_blocks)
        )

    def forward(self, x: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        for block, attn in zip(self.blocks, self.attns):
            x = attn(block(x, t))
        return x


class UNet(nn.Module):
    def __init__(self, config: UNetConfig):
        super().__init__()
        if config.fp8_history_skip_empty and not config.device_scale_history:
            raise ValueError("fp8_history_skip_empty needs device_scale_history")
        self.config = config
        self.base_channs = base = config.base_hidden
        chans = [s * base for s in config.scales]
        self.conv_in = nn.Conv2d(config.in_channels, chans[0], (3, 3), padding=1, bias=False)

        down, up = [], []
        res = config.in_resolution
        for cur, nxt in zip(chans[:-1], chans[1:]):
            attn = res in config.attn_resolutions
            down.append(Stage(config, cur, cur, nxt, attention=attn, num_blocks=config.n_resblocks))
            up.insert(0, Stage(config, 2 * nxt, cur, cur, attention=attn, num_blocks=config.n_resblocks + 1))
            res //= 2
        mid = chans[-1]
        down.append(Stage(config, mid, mid, mid, num_blocks=config.n_resblocks))
        up.insert(0, Stage(config, 2 * mid, mid, mid, num_blocks=config.n_resblocks + 1))
        # the reference always gives the middle stage attention (unet.py:311-318)
        self.mid = Stage(config, mid, mid, mid, attention=True, num_blocks=config.n_resblocks)
        self.down_stages = nn.ModuleList(down)
        self.up_stages = nn.ModuleList(up)

        self.out = nn.Sequential(
            nn.GroupNorm(32, chans[0]), nn.SiLU(),
            nn.Conv2d(chans[0], config.in_channels, (3, 3), padding=1, bias=False),
        )
        self.time_embed = nn.Sequential(
            nn.Linear(base, 4 * base, bias=False), nn.SiLU(), nn.Linear(4 * base, 4 * base, bias=False), nn.SiLU(),
        )
        nn.init.zeros_(self.out[-1].weight)
        half = base // 2
        freqs = torch.exp(-torch.arange(half, dtype=torch.float32) * (math.log(10000.0) / half))
        self.register_buffer("freqs", freqs, persistent=False)
        self._time_w16 = None  # bf16 time-MLP weights from the step's batched cast
        # every residual block's dropout seed in one device vector: one clone and one increment per
        # training step instead of one pair per block (advanced on the device, so a captured graph
        # draws new masks each replay)
        self._res_blocks = [m for m in self.modules() if isinstance(m, ResidualBlock)]
        self.register_buffer("dropout_seed", torch.randint(0, 2**62, (len(self._res_blocks),), dtype=torch.int64),
                             persistent=False)

    def _timestep(self, t: torch.Tensor) -> torch.Tensor:
        emb = t[:, None].float() * self.freqs[None]
        emb = torch.cat([emb.sin(), emb.cos()], dim=1)
        if self.base_channs % 2 == 1:
            emb = F.pad(emb, (0, 1))
        return emb

    def forward(self, x: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        cfg = self.config
        if cfg.fp8_convs_enabled and cfg.fp8_scaling_type == "delayed" and cfg.device_scale_history:
            # process-wide mode, read by the history-updating launches of this step (forward and backward)
            _lib.set_empty_tensor_history(1 if cfg.fp8_history_skip_empty else 0)
        # The weights of the delayed-scaling FP8 convs that ran last time are quantized in one batch
        # (identical bytes and histories to quantizing each inside its conv).
        batch = getattr(self, "_fp8_delayed_convs", None)
        if batch:
            quantize_conv_weights(batch)
        self._time_w16 = self._cast_bf16_weights() if self.config.batched_weight_cast else None
        if self.training and self.config.fused_norm and self._res_blocks:
            seeds = self.dropout_seed.clone()
            self.dropout_seed.add_(1)
            for i, b in enumerate(self._res_blocks):
                b._seed = seeds[i]
        out = self._forward(x, t)
        for b in self._res_blocks:
            b._seed = None
        convs = [m for m in self.modules() if isinstance(m, Conv2dFP8) and m.used_fp8_delayed]
        for m in convs:
            m.used_fp8_delayed = False
        for m in batch or ():
            m._pre_weight = None  # a conv that did not run must not keep this step's weights
        self._fp8_delayed_convs = convs if len(convs) <= 64 else None
        return out

    def _cast_bf16_weights(self):
        """One batched bf16 cast of the weights of the layers that run in bf16: each attention's
        (qkv, out), each 1x1 skip conv, and the time MLP (returned).  None when they would not be
        cast (autocast off, or any of them swapped for an FP8 layer)."""
        attns = [m for m in self.modules() if isinstance(m, CHWAttention)]
        skips = [m for m in self.modules() if isinstance(m, ResidualBlock) and isinstance(m.skip_connection, nn.Conv2d)]
        mlp = (self.time_embed[0], self.time_embed[2])
        lins = [lin for a in attns for lin in (a.qkv, a.out)] + list(mlp)
        if any(type(lin) is not nn.Linear for lin in lins):
            return None
        weights = [lin.weight for lin in lins] + [b.skip_connection.weight for b in skips]
        if not batch_cast_applies(weights):
            return None
        w16 = cast_weights_bf16(weights)
        for i, a in enumerate(attns):
            a._w16 = (w16[2 * i], w16[2 * i + 1])
        k = 2 * len(attns) + 2
        for b, w in zip(skips, w16[k:]):
            b._skip_w16 = w
        return w16[k - 2], w16[k - 1]

    def _batched_time_embeds(self, t_emb: torch.Tensor) -> None:
        """One GEMM for all blocks' ``t_embed_wb`` projections (same input); each block gets its column slice."""
        blocks = [m for m in self.modules() if isinstance(m, ResidualBlock)]
        weights = [b.t_embed_wb.mlp.weight for b in blocks]
        if self.config.batched_weight_cast and batch_cast_applies(weights) and all(w.is_contiguous() for w in weights):
            e = F.linear(t_emb, cast_cat_weights_bf16(weights))
        else:
            e = F.linear(t_emb, torch.cat(weights, dim=0))
        for b, part in zip(blocks, torch.split(e, [w.shape[0] for w in weights], dim=1)):
            b._emb = part[:, :, None, None]

    def _forward(self, x: torch.Tensor, t: torch.Tensor) -> torch.Tensor:
        w16, self._time_w16 = self._time_w16, None
        if w16 is None:
            t_emb = self.time_embed(self._timestep(t))
        else:  # time_embed = Linear, SiLU, Linear, SiLU on the batch-cast weights
            h = F.silu(F.linear(self._timestep(t), w16[0], self.time_embed[0].bias))
            t_emb = F.silu(F.linear(h, w16[1], self.time_embed[2].bias))
        if self.config.batched_time_embed:
            self._batched_time_embeds(t_emb)
        act = self.conv_in(x)
        skips = []
        fused = self.config.fused_resample
        for i, stage in enumerate(self.down_stages):
            if i > 0:
                act = downsample_nearest(act) if fused else F.interpolate(act, scale_factor=0.5, mode="nearest")
            act = stage(act, t_emb)
            skips.append(act)
        act = self.mid(act, t_emb)
        for i, stage in enumerate(self.up_stages):
            h = skips.pop()
            if fused:
                blk = stage.blocks[0]
                if self.config.fused_skip_cast and isinstance(blk.skip_connection, nn.Conv2d):
                    y, blk._skip_in = upsample_cat_pair(act, h, 2 if i > 0 else 1)
                else:
                    y = upsample_cat(act, h, 2 if i > 0 else 1)
                act = stage(y, t_emb)
            else:
                up = F.interpolate(act, scale_factor=2.0, mode="nearest") if i > 0 else act
                act = stage(torch.cat([up, h], dim=1), t_emb)
        if self.config.fused_norm and fused_norm_supported(act, self.out[0]):
            return self.out[2](group_norm_act(act, self.out[0]))
        return self.out(act)


def fp8_conv_modules(model: nn.Module) -> list[Conv2dFP8]:
    return [m for m in model.modules() if isinstance(m, Conv2dFP8)]


__all__ = ["UNetConfig", "UNet", "Conv2dFP8", "ResidualBlock", "CHWAttention", "Stage", "TimeEmbed",
           "fp8_conv_modules"]
