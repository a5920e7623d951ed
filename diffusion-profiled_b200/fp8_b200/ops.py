"""Torch custom ops over the C ABI (``fp8_b200::*``).

Each op allocates its outputs and workspaces with the torch caching allocator,
launches the native kernels on torch's current stream and never synchronises,
so the ops can be captured in CUDA graphs.  They are registered with
``torch.library.custom_op`` plus fake (meta) implementations so that
``torch.compile`` treats them as opaque nodes.

Layouts: 4-D activations and conv weights are channels_last (physically NHWC /
[Cout][3][3][Cin]); FP8 tensors are ``torch.float8_e4m3fn``; scales are fp32
0-d device tensors holding the dequantisation scale ``amax / 448``.
"""

from __future__ import annotations

import ctypes
from ctypes import c_int64, c_void_p

import torch

from . import _lib

FP8_DTYPE = torch.float8_e4m3fn

EPILOGUE_NONE = _lib.EPILOGUE_NONE
EPILOGUE_BIAS = _lib.EPILOGUE_BIAS
EPILOGUE_BIAS_SILU = _lib.EPILOGUE_BIAS_SILU


def _ptr(t: torch.Tensor | None) -> c_void_p:
    return c_void_p(0 if t is None else t.data_ptr())


def _stream(device: torch.device) -> c_void_p:
    return c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("fp8_b200 ops run on CUDA tensors only (there is no CPU path)")
        if t.device != dev:
            raise RuntimeError(f"tensors on different devices: {t.device} vs {dev}")
    return dev


def _nhwc_dims(t: torch.Tensor) -> tuple[int, int, int, int]:
    b, c, h, w = t.shape
    return b, c, h, w


# ----------------------------------------------------------------------------- quantize
@torch.library.custom_op("fp8_b200::quantize_current", mutates_args=())
def quantize_current(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-tensor e4m3 quantisation with the tensor's own amax (fp8_kernels.py:559-601)."""
    dev = _require_cuda(x)
    if x.dtype != torch.bfloat16:
        raise RuntimeError(f"quantize expects bfloat16, got {x.dtype}")
    if not (x.is_contiguous() or x.is_contiguous(memory_format=torch.channels_last)):
        raise RuntimeError("quantize expects a dense (contiguous or channels_last) tensor")
    q = torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.preserve_format)
    scale = torch.empty((), device=dev, dtype=torch.float32)
    n = x.numel()
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws_bytes = lib.fp8_quantize_workspace_bytes(n)
        ws = torch.empty(max(ws_bytes // 4, 1), device=dev, dtype=torch.float32)
        _lib.check(
            lib.fp8_quantize_current(_ptr(x), _ptr(q), _ptr(scale), _ptr(ws), ws.numel() * 4, n, _stream(dev)),
            "fp8_quantize_current",
        )
    return q, scale


@quantize_current.register_fake
def _(x):
    return torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.preserve_format), x.new_empty(
        (), dtype=torch.float32
    )


@torch.library.custom_op("fp8_b200::quantize_current_pair", mutates_args=())
def quantize_current_pair(x: torch.Tensor, w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor,
                                                                     torch.Tensor]:
    """quantize_current of two tensors (a layer's input and weight) in one amax and one
    cast launch -> (xq, sx, wq, sw); bytes and scales as two quantize_current calls."""
    dev = _require_cuda(x, w)
    for t in (x, w):
        if t.dtype != torch.bfloat16:
            raise RuntimeError(f"quantize expects bfloat16, got {t.dtype}")
        if not (t.is_contiguous() or t.is_contiguous(memory_format=torch.channels_last)):
            raise RuntimeError("quantize expects a dense (contiguous or channels_last) tensor")
    qs = [torch.empty_like(t, dtype=FP8_DTYPE, memory_format=torch.preserve_format) for t in (x, w)]
    scales = [torch.empty((), device=dev, dtype=torch.float32) for _ in range(2)]
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(max(lib.fp8_quantize_multi_workspace_bytes(2) // 4, 1), device=dev, dtype=torch.float32)
        xs = (c_void_p * 2)(x.data_ptr(), w.data_ptr())
        qp = (c_void_p * 2)(qs[0].data_ptr(), qs[1].data_ptr())
        sp = (c_void_p * 2)(scales[0].data_ptr(), scales[1].data_ptr())
        ns = (ctypes.c_int64 * 2)(x.numel(), w.numel())
        _lib.check(lib.fp8_quantize_current_multi(2, xs, qp, sp, ns, _ptr(ws), ws.numel() * 4, _stream(dev)),
                   "fp8_quantize_current_multi")
    return qs[0], scales[0], qs[1], scales[1]


@quantize_current_pair.register_fake
def _(x, w):
    return (torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.preserve_format), x.new_empty((), dtype=torch.float32),
            torch.empty_like(w, dtype=FP8_DTYPE, memory_format=torch.preserve_format), w.new_empty((), dtype=torch.float32))


@torch.library.custom_op("fp8_b200::quantize_delayed", mutates_args=())
def quantize_delayed(x: torch.Tensor, prev_scale: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Cast with ``prev_scale``; also return the scale of x's own amax (fp8_kernels.py:518-556)."""
    dev = _require_cuda(x, prev_scale)
    if x.dtype != torch.bfloat16:
        raise RuntimeError(f"quantize expects bfloat16, got {x.dtype}")
    if prev_scale.dtype != torch.float32 or prev_scale.numel() != 1:
        raise RuntimeError("prev_scale must be a one-element float32 tensor")
    if not (x.is_contiguous() or x.is_contiguous(memory_format=torch.channels_last)):
        raise RuntimeError("quantize expects a dense (contiguous or channels_last) tensor")
    q = torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.preserve_format)
    scale = torch.empty((), device=dev, dtype=torch.float32)
    n = x.numel()
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws_bytes = lib.fp8_quantize_workspace_bytes(n)
        ws = torch.empty(max(ws_bytes // 4, 1), device=dev, dtype=torch.float32)
        _lib.check(
            lib.fp8_quantize_delayed(
                _ptr(x), _ptr(q), _ptr(prev_scale), _ptr(scale), _ptr(ws), ws.numel() * 4, n, _stream(dev)
            ),
            "fp8_quantize_delayed",
        )
    return q, scale


@quantize_delayed.register_fake
def _(x, prev_scale):
    return torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.preserve_format), x.new_empty(
        (), dtype=torch.float32
    )


def _check_window(window: torch.Tensor, pos: torch.Tensor, dev: torch.device) -> None:
    if window.device != dev or window.dtype != torch.float32 or window.dim() != 1 or not window.is_contiguous():
        raise RuntimeError("the scale history must be a contiguous 1-D float32 tensor on the input's device")
    if pos.device != dev or pos.dtype != torch.int64 or pos.numel() != 1:
        raise RuntimeError("the history position must be a one-element int64 tensor on the input's device")


@torch.library.custom_op("fp8_b200::quantize_delayed_window", mutates_args=("window", "pos"))
def quantize_delayed_window(x: torch.Tensor, window: torch.Tensor, pos: torch.Tensor,
                            advance: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Delayed cast with the scale history on the device -> (e4m3, scale used).

    Casts with ``max(window)`` (the reference module's ``torch.max(amax_window)``),
    then stores this tensor's own scale at ``window[pos]`` and, if ``advance``,
    steps ``pos`` (unet.py:69-91).  Bit for bit ``quantize_delayed(x, window.max())``
    followed by the module's scatter / position update."""
    dev = _require_cuda(x, window, pos)
    if x.dtype != torch.bfloat16:
        raise RuntimeError(f"quantize expects bfloat16, got {x.dtype}")
    if not (x.is_contiguous() or x.is_contiguous(memory_format=torch.channels_last)):
        raise RuntimeError("quantize expects a dense (contiguous or channels_last) tensor")
    _check_window(window, pos, dev)
    q = torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.preserve_format)
    used = torch.empty((), device=dev, dtype=torch.float32)
    n = x.numel()
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(max(lib.fp8_quantize_workspace_bytes(n) // 4, 1), device=dev, dtype=torch.float32)
        _lib.check(lib.fp8_quantize_delayed_window(
            _ptr(x), _ptr(q), _ptr(window), window.numel(), _ptr(pos), int(advance), _ptr(used), _ptr(ws),
            ws.numel() * 4, n, _stream(dev)), "fp8_quantize_delayed_window")
    return q, used


@quantize_delayed_window.register_fake
def _(x, window, pos, advance):
    return (torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.preserve_format),
            x.new_empty((), dtype=torch.float32))


@torch.library.custom_op("fp8_b200::quantize_weights_delayed", mutates_args=("windows",))
def quantize_weights_delayed(weights: list[torch.Tensor], windows: list[torch.Tensor],
                             positions: list[torch.Tensor]) -> list[torch.Tensor]:
    """Delayed quantize of many fp32 weights in three launches -> [q_0 .. q_{n-1}, scale_0 .. scale_{n-1}].

    Weight t is rounded to bf16, cast with ``max(windows[t])`` (returned as scale_t) and its own scale
    stored at ``windows[t][positions[t]]``; positions are not advanced (the activation quantize of the
    same module does that).  Bytes equal ``quantize_delayed_window(weights[t].bfloat16(), ...)``."""
    count = len(weights)
    if count == 0 or len(windows) != count or len(positions) != count:
        raise RuntimeError("weights, windows and positions must be non-empty lists of one length")
    dev = _require_cuda(*weights)
    lens = {int(w.numel()) for w in windows}
    if len(lens) != 1:
        raise RuntimeError("all scale histories must have one length")
    for w, win, pos in zip(weights, windows, positions):
        if w.dtype != torch.float32 or not (w.is_contiguous() or w.is_contiguous(memory_format=torch.channels_last)):
            raise RuntimeError("weights must be dense float32 tensors")
        _check_window(win, pos, dev)
    qs = [torch.empty_like(w, dtype=FP8_DTYPE, memory_format=torch.preserve_format) for w in weights]
    used = [torch.empty((), device=dev, dtype=torch.float32) for _ in weights]
    arr = lambda ts: (c_void_p * count)(*[t.data_ptr() for t in ts])  # noqa: E731
    n = (c_int64 * count)(*[w.numel() for w in weights])
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(max(lib.fp8_quantize_weights_delayed_workspace_bytes(count, n) // 4, 1), device=dev,
                         dtype=torch.float32)
        _lib.check(lib.fp8_quantize_weights_delayed(
            count, arr(weights), arr(qs), n, arr(windows), lens.pop(), arr(positions), arr(used), _ptr(ws),
            ws.numel() * 4, _stream(dev)), "fp8_quantize_weights_delayed")
    return qs + used


@quantize_weights_delayed.register_fake
def _(weights, windows, positions):
    return ([torch.empty_like(w, dtype=FP8_DTYPE, memory_format=torch.preserve_format) for w in weights]
            + [w.new_empty((), dtype=torch.float32) for w in weights])


# ----------------------------------------------------------------------------- batched casts
def _cast_call(srcs: list[torch.Tensor], dsts: list[torch.Tensor], to_bf16: bool, dev: torch.device) -> None:
    lib = _lib.load()
    with torch.cuda.device(dev):
        for i in range(0, len(srcs), 64):  # fp8_cast_batch takes 64 tensors per call
            s, d = srcs[i:i + 64], dsts[i:i + 64]
            k = len(s)
            _lib.check(lib.fp8_cast_batch(k, (c_void_p * k)(*[t.data_ptr() for t in s]),
                                          (c_void_p * k)(*[t.data_ptr() for t in d]),
                                          (c_int64 * k)(*[t.numel() for t in s]), int(to_bf16), _stream(dev)),
                       "fp8_cast_batch")


def _dense(t: torch.Tensor) -> bool:
    return t.is_contiguous() or (t.dim() == 4 and t.is_contiguous(memory_format=torch.channels_last))


@torch.library.custom_op("fp8_b200::cast_batch", mutates_args=())
def cast_batch(srcs: list[torch.Tensor], to_bf16: bool) -> list[torch.Tensor]:
    """Each tensor cast fp32 -> bf16 (``to_bf16``) or bf16 -> fp32, same shape and strides, in one
    launch per 64 tensors: the values of ``t.to(dtype)``."""
    if not srcs:
        return []
    dev = _require_cuda(*srcs)
    want = torch.float32 if to_bf16 else torch.bfloat16
    for t in srcs:
        if t.dtype != want or not _dense(t):
            raise RuntimeError(f"cast_batch expects dense {want} tensors")
    dst_dt = torch.bfloat16 if to_bf16 else torch.float32
    dsts = [torch.empty_like(t, dtype=dst_dt) for t in srcs]
    _cast_call(srcs, dsts, to_bf16, dev)
    return dsts


@cast_batch.register_fake
def _(srcs, to_bf16):
    return [torch.empty_like(t, dtype=torch.bfloat16 if to_bf16 else torch.float32) for t in srcs]


@torch.library.custom_op("fp8_b200::cast_cat_bf16", mutates_args=())
def cast_cat_bf16(srcs: list[torch.Tensor]) -> torch.Tensor:
    """``torch.cat(srcs, dim=0).to(torch.bfloat16)`` for contiguous 2-D fp32 tensors of one width,
    written directly (one launch, no fp32 concatenation)."""
    dev = _require_cuda(*srcs)
    cols = srcs[0].shape[1] if srcs and srcs[0].dim() == 2 else -1
    for t in srcs:
        if t.dtype != torch.float32 or t.dim() != 2 or t.shape[1] != cols or not t.is_contiguous():
            raise RuntimeError("cast_cat_bf16 expects contiguous 2-D float32 tensors of one width")
    out = torch.empty((sum(t.shape[0] for t in srcs), cols), device=dev, dtype=torch.bfloat16)
    _cast_call(srcs, list(torch.split(out, [t.shape[0] for t in srcs], dim=0)), True, dev)
    return out


@cast_cat_bf16.register_fake
def _(srcs):
    return srcs[0].new_empty((sum(t.shape[0] for t in srcs), srcs[0].shape[1]), dtype=torch.bfloat16)


# ----------------------------------------------------------------------------- transposes
@torch.library.custom_op("fp8_b200::transpose_2d", mutates_args=())
def transpose_2d(src: torch.Tensor) -> torch.Tensor:
    """[R, C] -> [C, R] byte transpose (fp8_kernels.py:321-337)."""
    dev = _require_cuda(src)
    if src.dim() != 2 or not src.is_contiguous() or src.element_size() != 1:
        raise RuntimeError("transpose_2d expects a contiguous 2-D 1-byte tensor")
    rows, cols = src.shape
    dst = torch.empty((cols, rows), device=dev, dtype=src.dtype)
    with torch.cuda.device(dev):
        _lib.call("fp8_transpose_2d", _ptr(src), _ptr(dst), rows, cols, _stream(dev))
    return dst


@transpose_2d.register_fake
def _(src):
    return src.new_empty((src.shape[1], src.shape[0]))


# ----------------------------------------------------------------------------- conv 3x3
def _check_conv_operand(t: torch.Tensor, name: str) -> None:
    if t.dim() != 4:
        raise RuntimeError(f"{name} must be 4-D")
    if t.dtype != FP8_DTYPE:
        raise RuntimeError(f"{name} must be float8_e4m3fn, got {t.dtype}")
    if not t.is_contiguous(memory_format=torch.channels_last):
        raise RuntimeError(f"{name} must be channels_last contiguous")


def _check_scale(s: torch.Tensor, dev: torch.device, name: str) -> None:
    if s.device != dev or s.dtype != torch.float32 or s.numel() != 1:
        raise RuntimeError(f"{name} must be a one-element float32 tensor on {dev}")


@torch.library.custom_op("fp8_b200::conv3x3_fwd", mutates_args=())
def conv3x3_fwd(
    xq: torch.Tensor,
    wq: torch.Tensor,
    sx: torch.Tensor,
    sw: torch.Tensor,
    bias: torch.Tensor | None = None,
    epilogue: int = EPILOGUE_NONE,
) -> torch.Tensor:
    """bf16 channels_last ``conv2d(xq*sx, wq*sw, padding=1)`` (+bias, +SiLU)."""
    dev = _require_cuda(xq, wq)
    _check_conv_operand(xq, "x")
    _check_conv_operand(wq, "weight")
    _check_scale(sx, dev, "x_scale")
    _check_scale(sw, dev, "weight_scale")
    b, cin, h, w = xq.shape
    cout = wq.shape[0]
    if tuple(wq.shape[1:]) != (cin, 3, 3):
        raise RuntimeError(f"weight shape {tuple(wq.shape)} does not match Cin={cin} 3x3")
    if epilogue != EPILOGUE_NONE:
        if bias is None or bias.dtype != torch.bfloat16 or bias.numel() != cout or not bias.is_contiguous():
            raise RuntimeError("bias epilogue needs a contiguous bf16 bias of Cout elements")
    y = torch.empty((b, cout, h, w), device=dev, dtype=torch.bfloat16, memory_format=torch.channels_last)
    with torch.cuda.device(dev):
        _lib.call(
            "fp8_conv3x3_fwd", _ptr(xq), _ptr(wq), _ptr(y), _ptr(sx), _ptr(sw), _ptr(bias), epilogue, b, h, w,
            cin, cout, _stream(dev),
        )
    return y


@conv3x3_fwd.register_fake
def _(xq, wq, sx, sw, bias=None, epilogue=EPILOGUE_NONE):
    b, _, h, w = xq.shape
    return torch.empty(
        (b, wq.shape[0], h, w), device=xq.device, dtype=torch.bfloat16, memory_format=torch.channels_last
    )


@torch.library.custom_op("fp8_b200::conv3x3_dgrad", mutates_args=())
def conv3x3_dgrad(dyq: torch.Tensor, wq: torch.Tensor, sdy: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """bf16 channels_last input gradient of the 3x3 conv (fp8_kernels.py:671-709)."""
    dev = _require_cuda(dyq, wq)
    _check_conv_operand(dyq, "dy")
    _check_conv_operand(wq, "weight")
    _check_scale(sdy, dev, "dy_scale")
    _check_scale(sw, dev, "weight_scale")
    b, cout, h, w = dyq.shape
    cin = wq.shape[1]
    if tuple(wq.shape) != (cout, cin, 3, 3):
        raise RuntimeError(f"weight shape {tuple(wq.shape)} does not match Cout={cout} 3x3")
    dx = torch.empty((b, cin, h, w), device=dev, dtype=torch.bfloat16, memory_format=torch.channels_last)
    with torch.cuda.device(dev):
        # The weights are read in place where the kernel allows it (no workspace);
        # otherwise the library re-lays them out to [Cin][3][3][Cout] in the workspace.
        ws_bytes = _lib.load().fp8_conv3x3_dgrad_w_workspace_bytes(b, h, w, cin, cout)
        ws = torch.empty((ws_bytes,), device=dev, dtype=torch.uint8) if ws_bytes else None
        _lib.call(
            "fp8_conv3x3_dgrad_w", _ptr(dyq), _ptr(wq), _ptr(dx), _ptr(sdy), _ptr(sw), b, h, w, cin, cout,
            _ptr(ws), ws_bytes, _stream(dev),
        )
    return dx


@conv3x3_dgrad.register_fake
def _(dyq, wq, sdy, sw):
    b, _, h, w = dyq.shape
    return torch.empty(
        (b, wq.shape[1], h, w), device=dyq.device, dtype=torch.bfloat16, memory_format=torch.channels_last
    )


def dgrad_needs_relayout(b: int, h: int, w: int, cin: int, cout: int) -> bool:
    """Whether conv3x3_dgrad re-lays the weights out for this geometry (else it reads them in place)."""
    return _lib.load().fp8_conv3x3_dgrad_w_workspace_bytes(b, h, w, cin, cout) > 0


@torch.library.custom_op("fp8_b200::transpose_conv_weights", mutates_args=())
def transpose_conv_weights(wqs: list[torch.Tensor]) -> list[torch.Tensor]:
    """Each e4m3 channels_last weight [Cout, Cin, 3, 3] re-laid out as [Cin][3][3][Cout] (a contiguous
    [Cin, 9*Cout] tensor, the data-grad's B operand), in one launch per 64 weights."""
    if not wqs:
        return []
    dev = _require_cuda(*wqs)
    for t in wqs:
        _check_conv_operand(t, "weight")
    outs = [torch.empty((t.shape[1], 9 * t.shape[0]), device=dev, dtype=FP8_DTYPE) for t in wqs]
    lib = _lib.load()
    with torch.cuda.device(dev):
        for i in range(0, len(wqs), 64):
            src, dst = wqs[i:i + 64], outs[i:i + 64]
            k = len(src)
            _lib.check(lib.fp8_conv_weight_transpose_batch(
                k, (c_void_p * k)(*[t.data_ptr() for t in src]), (c_void_p * k)(*[t.data_ptr() for t in dst]),
                (ctypes.c_int * k)(*[t.shape[0] for t in src]), (ctypes.c_int * k)(*[t.shape[1] for t in src]),
                _stream(dev)), "fp8_conv_weight_transpose_batch")
    return outs


@transpose_conv_weights.register_fake
def _(wqs):
    return [t.new_empty((t.shape[1], 9 * t.shape[0])) for t in wqs]


@torch.library.custom_op("fp8_b200::conv3x3_dgrad_pre", mutates_args=())
def conv3x3_dgrad_pre(dyq: torch.Tensor, wq_t: torch.Tensor, sdy: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """conv3x3_dgrad with the weights already re-laid out by transpose_conv_weights ([Cin, 9*Cout])."""
    dev = _require_cuda(dyq, wq_t)
    _check_conv_operand(dyq, "dy")
    _check_scale(sdy, dev, "dy_scale")
    _check_scale(sw, dev, "weight_scale")
    b, cout, h, w = dyq.shape
    if wq_t.dtype != FP8_DTYPE or wq_t.dim() != 2 or not wq_t.is_contiguous() or wq_t.shape[1] != 9 * cout:
        raise RuntimeError("wq_t must be a contiguous [Cin, 9*Cout] float8_e4m3fn tensor")
    cin = wq_t.shape[0]
    dx = torch.empty((b, cin, h, w), device=dev, dtype=torch.bfloat16, memory_format=torch.channels_last)
    with torch.cuda.device(dev):
        _lib.call("fp8_conv3x3_dgrad", _ptr(dyq), _ptr(wq_t), _ptr(dx), _ptr(sdy), _ptr(sw), b, h, w, cin, cout,
                  _stream(dev))
    return dx


@conv3x3_dgrad_pre.register_fake
def _(dyq, wq_t, sdy, sw):
    b, _, h, w = dyq.shape
    return torch.empty((b, wq_t.shape[0], h, w), device=dyq.device, dtype=torch.bfloat16,
                       memory_format=torch.channels_last)


@torch.library.custom_op("fp8_b200::conv3x3_wgrad", mutates_args=())
def conv3x3_wgrad(
    xq: torch.Tensor, dyq: torch.Tensor, sx: torch.Tensor, sdy: torch.Tensor, split_k: int = 0, widen: bool = False
) -> torch.Tensor:
    """bf16 channels_last weight gradient [Cout, Cin, 3, 3] (fp8_kernels.py:723-808).

    ``widen=True``: the same bf16 values stored as fp32, which is what an fp32 weight's
    gradient becomes when autograd casts the bf16 result (fp8_kernels.py:875-913) to the
    weight's dtype -- written by the reduce pass itself, with no cast launch."""
    dev = _require_cuda(xq, dyq)
    _check_conv_operand(xq, "x")
    _check_conv_operand(dyq, "dy")
    _check_scale(sx, dev, "x_scale")
    _check_scale(sdy, dev, "dy_scale")
    b, cin, h, w = xq.shape
    cout = dyq.shape[1]
    if (dyq.shape[0], dyq.shape[2], dyq.shape[3]) != (b, h, w):
        raise RuntimeError("x and dy batch/spatial dims differ")
    dt = torch.float32 if widen else torch.bfloat16
    dw = torch.empty((cout, cin, 3, 3), device=dev, dtype=dt, memory_format=torch.channels_last)
    lib = _lib.load()
    fn = "fp8_conv3x3_wgrad_f32" if widen else "fp8_conv3x3_wgrad"
    with torch.cuda.device(dev):
        ws_bytes = lib.fp8_conv3x3_wgrad_workspace_bytes(b, h, w, cin, cout, split_k)
        ws = torch.empty(max(ws_bytes // 4, 4), device=dev, dtype=torch.float32)
        _lib.check(
            getattr(lib, fn)(
                _ptr(xq), _ptr(dyq), _ptr(dw), _ptr(sx), _ptr(sdy), b, h, w, cin, cout, split_k, _ptr(ws),
                ws.numel() * 4, _stream(dev),
            ),
            fn,
        )
    return dw


@conv3x3_wgrad.register_fake
def _(xq, dyq, sx, sdy, split_k=0, widen=False):
    return torch.empty(
        (dyq.shape[1], xq.shape[1], 3, 3), device=xq.device, dtype=torch.float32 if widen else torch.bfloat16,
        memory_format=torch.channels_last
    )


# Per-device side stream of conv3x3_backward (the weight gradient runs there beside the data
# gradient).  Created on first use outside a CUDA-graph capture; while a capture is in progress
# and none exists yet, the two gradients run one after the other on the current stream.
_SIDE_STREAMS: dict[int, torch.cuda.Stream] = {}


def _side_stream(dev: torch.device) -> torch.cuda.Stream | None:
    s = _SIDE_STREAMS.get(dev.index)
    if s is None and not torch.cuda.is_current_stream_capturing():
        s = _SIDE_STREAMS[dev.index] = torch.cuda.Stream(dev)
    return s


@torch.library.custom_op("fp8_b200::conv3x3_backward", mutates_args=())
def conv3x3_backward(
    dyq: torch.Tensor, wq: torch.Tensor, sdy: torch.Tensor, sw: torch.Tensor, xq: torch.Tensor, sx: torch.Tensor,
    split_k: int = 0, widen: bool = False, wq_t: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """(dx, dw) of the 3x3 conv: conv3x3_dgrad (or conv3x3_dgrad_pre with ``wq_t``) and
    conv3x3_wgrad, the same results, with the weight gradient launched on a side stream so
    that it overlaps the data gradient (the two are independent given the e4m3 operands; the
    reference computes them one after the other, fp8_kernels.py:875-913).  Outputs and
    workspaces are allocated on the current stream before the fork, and the current stream
    waits for the side stream before the op returns, so callers see ordinary stream order."""
    dev = _require_cuda(dyq, wq, xq)
    _check_conv_operand(dyq, "dy")
    _check_conv_operand(xq, "x")
    _check_scale(sdy, dev, "dy_scale")
    _check_scale(sw, dev, "weight_scale")
    _check_scale(sx, dev, "x_scale")
    b, cout, h, w = dyq.shape
    cin = xq.shape[1]
    if (xq.shape[0], xq.shape[2], xq.shape[3]) != (b, h, w):
        raise RuntimeError("x and dy batch/spatial dims differ")
    if wq_t is None:
        _check_conv_operand(wq, "weight")
        if tuple(wq.shape) != (cout, cin, 3, 3):
            raise RuntimeError(f"weight shape {tuple(wq.shape)} does not match Cout={cout} Cin={cin} 3x3")
    elif wq_t.dtype != FP8_DTYPE or tuple(wq_t.shape) != (cin, 9 * cout) or not wq_t.is_contiguous():
        raise RuntimeError("wq_t must be a contiguous [Cin, 9*Cout] float8_e4m3fn tensor")
    lib = _lib.load()
    dx = torch.empty((b, cin, h, w), device=dev, dtype=torch.bfloat16, memory_format=torch.channels_last)
    dw = torch.empty((cout, cin, 3, 3), device=dev, dtype=torch.float32 if widen else torch.bfloat16,
                     memory_format=torch.channels_last)
    with torch.cuda.device(dev):
        ws_w_bytes = lib.fp8_conv3x3_wgrad_workspace_bytes(b, h, w, cin, cout, split_k)
        ws_w = torch.empty(max(ws_w_bytes // 4, 4), device=dev, dtype=torch.float32)
        ws_d_bytes = lib.fp8_conv3x3_dgrad_w_workspace_bytes(b, h, w, cin, cout) if wq_t is None else 0
        ws_d = torch.empty((ws_d_bytes,), device=dev, dtype=torch.uint8) if ws_d_bytes else None
        cur = torch.cuda.current_stream(dev)
        side = _side_stream(dev)
        if side is not None:
            side.wait_stream(cur)
        fn = "fp8_conv3x3_wgrad_f32" if widen else "fp8_conv3x3_wgrad"
        _lib.check(
            getattr(lib, fn)(
                _ptr(xq), _ptr(dyq), _ptr(dw), _ptr(sx), _ptr(sdy), b, h, w, cin, cout, split_k, _ptr(ws_w),
                ws_w.numel() * 4, c_void_p((side if side is not None else cur).cuda_stream),
            ),
            fn,
        )
        if wq_t is None:
            _lib.call("fp8_conv3x3_dgrad_w", _ptr(dyq), _ptr(wq), _ptr(dx), _ptr(sdy), _ptr(sw), b, h, w, cin, cout,
                      _ptr(ws_d), ws_d_bytes, _stream(dev))
        else:
            _lib.call("fp8_conv3x3_dgrad", _ptr(dyq), _ptr(wq_t), _ptr(dx), _ptr(sdy), _ptr(sw), b, h, w, cin, cout,
                      _stream(dev))
        if side is not None:
            cur.wait_stream(side)
    return dx, dw


@conv3x3_backward.register_fake
def _(dyq, wq, sdy, sw, xq, sx, split_k=0, widen=False, wq_t=None):
    b, cout, h, w = dyq.shape
    cin = xq.shape[1]
    dx = torch.empty((b, cin, h, w), device=dyq.device, dtype=torch.bfloat16, memory_format=torch.channels_last)
    dw = torch.empty((cout, cin, 3, 3), device=dyq.device, dtype=torch.float32 if widen else torch.bfloat16,
                     memory_format=torch.channels_last)
    return dx, dw


# ----------------------------------------------------------------------------- GEMM (linear)
def _check_2d_fp8(t: torch.Tensor, name: str) -> None:
    if t.dim() != 2 or t.dtype != FP8_DTYPE or not t.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous 2-D float8_e4m3fn tensor")


@torch.library.custom_op("fp8_b200::gemm", mutates_args=())
def gemm(
    a: torch.Tensor,
    b: torch.Tensor,
    sa: torch.Tensor,
    sb: torch.Tensor,
    bias: torch.Tensor | None = None,
    epilogue: int = EPILOGUE_NONE,
) -> torch.Tensor:
    """``out[M, N] = (a[M, K] @ b[N, K].T) * sa * sb`` (+bias, +SiLU), bf16."""
    dev = _require_cuda(a, b)
    _check_2d_fp8(a, "a")
    _check_2d_fp8(b, "b")
    _check_scale(sa, dev, "a_scale")
    _check_scale(sb, dev, "b_scale")
    m, k = a.shape
    n = b.shape[0]
    if b.shape[1] != k:
        raise RuntimeError(f"inner dims differ: a {tuple(a.shape)} b {tuple(b.shape)}")
    if epilogue != EPILOGUE_NONE:
        if bias is None or bias.dtype != torch.bfloat16 or bias.numel() != n or not bias.is_contiguous():
            raise RuntimeError("bias epilogue needs a contiguous bf16 bias of N elements")
    out = torch.empty((m, n), device=dev, dtype=torch.bfloat16)
    with torch.cuda.device(dev):
        _lib.call(
            "fp8_gemm", _ptr(a), _ptr(b), _ptr(out), _ptr(sa), _ptr(sb), _ptr(bias), epilogue, m, n, k,
            _stream(dev),
        )
    return out


@gemm.register_fake
def _(a, b, sa, sb, bias=None, epilogue=EPILOGUE_NONE):
    return a.new_empty((a.shape[0], b.shape[0]), dtype=torch.bfloat16)


@torch.library.custom_op("fp8_b200::gemm_wgrad", mutates_args=())
def gemm_wgrad(dy: torch.Tensor, x: torch.Tensor, sdy: torch.Tensor, sx: torch.Tensor, split_k: int = 0) -> torch.Tensor:
    """``dw[N, K] = dy[M, N].T @ x[M, K] * sdy * sx`` in bf16."""
    dev = _require_cuda(dy, x)
    _check_2d_fp8(dy, "dy")
    _check_2d_fp8(x, "x")
    _check_scale(sdy, dev, "dy_scale")
    _check_scale(sx, dev, "x_scale")
    m, n = dy.shape
    if x.shape[0] != m:
        raise RuntimeError("dy and x row counts differ")
    k = x.shape[1]
    dw = torch.empty((n, k), device=dev, dtype=torch.bfloat16)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws_bytes = lib.fp8_gemm_wgrad_workspace_bytes(m, n, k, split_k)
        ws = torch.empty(max(ws_bytes // 4, 4), device=dev, dtype=torch.float32)
        _lib.check(
            lib.fp8_gemm_wgrad(
                _ptr(dy), _ptr(x), _ptr(dw), _ptr(sdy), _ptr(sx), m, n, k, split_k, _ptr(ws), ws.numel() * 4,
                _stream(dev),
            ),
            "fp8_gemm_wgrad",
        )
    return dw


@gemm_wgrad.register_fake
def _(dy, x, sdy, sx, split_k=0):
    return dy.new_empty((dy.shape[1], x.shape[1]), dtype=torch.bfloat16)


def device_error(device: torch.device | None = None) -> int:
    """Read and clear the device error word (synchronises the current stream)."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(dev):
        return _lib.device_error(torch.cuda.current_stream(dev).cuda_stream)


__all__ = [
    "FP8_DTYPE",
    "EPILOGUE_NONE",
    "EPILOGUE_BIAS",
    "EPILOGUE_BIAS_SILU",
    "quantize_current",
    "quantize_delayed",
    "transpose_2d",
    "conv3x3_fwd",
    "conv3x3_dgrad",
    "conv3x3_wgrad",
    "conv3x3_backward",
    "gemm",
    "gemm_wgrad",
    "device_error",
]


# ----------------------------------------------------------------------------- group norm + activation
def _gn_check(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, film: torch.Tensor | None,
              groups: int) -> tuple[int, int, int]:
    if x.dtype not in (torch.bfloat16, torch.float32) or x.dim() != 4 or not x.is_contiguous(
            memory_format=torch.channels_last):
        raise RuntimeError("group norm expects a channels_last bfloat16 or float32 [N, C, H, W] tensor")
    n, c, h, w = x.shape
    if gamma.dtype != torch.float32 or beta.dtype != torch.float32 or gamma.numel() != c or beta.numel() != c:
        raise RuntimeError("gamma / beta must be float32 [C]")
    if film is not None and (film.dtype != torch.bfloat16 or film.dim() != 2 or tuple(film.shape) != (n, 2 * c)
                             or film.stride(1) != 1 or film.stride(0) < 2 * c):
        raise RuntimeError("film must be a bfloat16 [N, 2C] (scale, shift) tensor with unit column stride")
    return n, c, h * w


def _film_ld(film: torch.Tensor | None, c: int) -> int:
    """Row pitch of the FiLM rows (they may be a column slice of all blocks' projections)."""
    return 2 * c if film is None else film.stride(0)


@torch.library.custom_op("fp8_b200::gn_act_fwd", mutates_args=())
def gn_act_fwd(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, film: torch.Tensor | None,
               seed: torch.Tensor | None, p: float, eps: float, groups: int) -> tuple[torch.Tensor, torch.Tensor]:
    """a = dropout(silu((film_scale + 1) * GroupNorm(x) + film_shift)) -> (a bf16 channels_last, stats [N, 2, G]).

    x is bf16 or fp32 (the dtype the reference's GroupNorm sees at that point).

    No reference kernel: replaces the torch chain of the reference ResBlock
    (unet.py:151, :157-159).  `seed` (int64 device scalar) selects the dropout mask."""
    dev = _require_cuda(x, gamma, beta)
    n, c, hw = _gn_check(x, gamma, beta, film, groups)
    out = torch.empty_like(x, dtype=torch.bfloat16, memory_format=torch.channels_last)
    stats = torch.empty((n, 2, groups), device=dev, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(max(lib.fp8_gn_workspace_bytes(n, hw, c) // 4, 4), device=dev, dtype=torch.float32)
        _lib.check(lib.fp8_gn_act_fwd(
            _ptr(x), int(x.dtype == torch.float32), _ptr(gamma), _ptr(beta), _ptr(film), _film_ld(film, c), _ptr(seed), float(p), float(eps), _ptr(stats),
            _ptr(out), n, hw, c, groups, _ptr(ws), ws.numel() * 4, _stream(dev)), "fp8_gn_act_fwd")
    return out, stats


@gn_act_fwd.register_fake
def _(x, gamma, beta, film, seed, p, eps, groups):
    return (torch.empty_like(x, dtype=torch.bfloat16, memory_format=torch.channels_last),
            x.new_empty((x.shape[0], 2, groups), dtype=torch.float32))


def _ln_check(x: torch.Tensor, gamma: torch.Tensor) -> tuple[int, int]:
    if x.dtype not in (torch.bfloat16, torch.float32) or not x.is_contiguous():
        raise RuntimeError("layer norm expects a contiguous bfloat16 or float32 tensor")
    c = x.shape[-1]
    if gamma.dtype != torch.float32 or gamma.shape != (c,):
        raise RuntimeError(f"layer-norm weight must be float32 [{c}]")
    return x.numel() // max(c, 1), c


@torch.library.custom_op("fp8_b200::layer_norm_fwd", mutates_args=())
def layer_norm_fwd(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                   eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """LayerNorm over the last dim -> (bf16 y, fp32 [tokens, 2] mean / rstd); nn.LayerNorm of unet.py:174."""
    dev = _require_cuda(x, gamma, beta)
    tokens, c = _ln_check(x, gamma)
    y = torch.empty(x.shape, device=dev, dtype=torch.bfloat16)
    mr = torch.empty((tokens, 2), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        _lib.call("fp8_layer_norm_fwd", _ptr(x), int(x.dtype == torch.float32), _ptr(gamma), _ptr(beta), float(eps),
                  _ptr(y), _ptr(mr), tokens, c, _stream(dev))
    return y, mr


@layer_norm_fwd.register_fake
def _(x, gamma, beta, eps):
    return x.new_empty(x.shape, dtype=torch.bfloat16), x.new_empty((x.numel() // x.shape[-1], 2), dtype=torch.float32)


@torch.library.custom_op("fp8_b200::layer_norm_bwd", mutates_args=())
def layer_norm_bwd(x: torch.Tensor, dy: torch.Tensor, gamma: torch.Tensor,
                   mean_rstd: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Backward of layer_norm_fwd -> (dx in x's dtype, dgamma, dbeta)."""
    dev = _require_cuda(x, dy, gamma, mean_rstd)
    tokens, c = _ln_check(x, gamma)
    dy = dy.to(torch.bfloat16).contiguous()
    if dy.shape != x.shape:
        raise RuntimeError("dy must be shaped like x")
    dx = torch.empty_like(x)
    dgamma = torch.empty((c,), device=dev, dtype=torch.float32)
    dbeta = torch.empty((c,), device=dev, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws_bytes = lib.fp8_layer_norm_workspace_bytes(tokens, c)
        ws = torch.empty((max(ws_bytes // 4, 4),), device=dev, dtype=torch.float32)
        _lib.check(lib.fp8_layer_norm_bwd(
            _ptr(x), int(x.dtype == torch.float32), _ptr(dy), _ptr(gamma), _ptr(mean_rstd), _ptr(dx), _ptr(dgamma),
            _ptr(dbeta), tokens, c, _ptr(ws), ws.numel() * 4, _stream(dev)), "fp8_layer_norm_bwd")
    return dx, dgamma, dbeta


@layer_norm_bwd.register_fake
def _(x, dy, gamma, mean_rstd):
    c = x.shape[-1]
    return torch.empty_like(x), x.new_empty((c,), dtype=torch.float32), x.new_empty((c,), dtype=torch.float32)


_DT = {torch.bfloat16: 0, torch.float32: 1}


def _resample_check(t: torch.Tensor, name: str) -> None:
    if t.dtype not in _DT or t.dim() != 4 or not t.is_contiguous(memory_format=torch.channels_last):
        raise RuntimeError(f"{name} must be a channels_last bfloat16 / float32 NCHW tensor")


@torch.library.custom_op("fp8_b200::resample_down2", mutates_args=())
def resample_down2(x: torch.Tensor) -> torch.Tensor:
    """Nearest downsampling by 2 -> fp32 (F.interpolate(scale_factor=0.5) under bf16 autocast, unet.py:368)."""
    dev = _require_cuda(x)
    _resample_check(x, "x")
    n, c, h, w = x.shape
    y = torch.empty((n, c, h // 2, w // 2), device=dev, dtype=torch.float32, memory_format=torch.channels_last)
    with torch.cuda.device(dev):
        _lib.call("fp8_resample_down2", _ptr(x), _DT[x.dtype], _ptr(y), n, h, w, c, _stream(dev))
    return y


@resample_down2.register_fake
def _(x):
    n, c, h, w = x.shape
    return x.new_empty((n, c, h // 2, w // 2), dtype=torch.float32).contiguous(memory_format=torch.channels_last)


@torch.library.custom_op("fp8_b200::resample_down2_bwd", mutates_args=())
def resample_down2_bwd(dy: torch.Tensor, h: int, w: int, x_fp32: bool) -> torch.Tensor:
    """Gradient of resample_down2: dy at the even pixels, zeros elsewhere, in the input's dtype."""
    dev = _require_cuda(dy)
    dy = dy.float().contiguous(memory_format=torch.channels_last)
    n, c = dy.shape[0], dy.shape[1]
    dt = torch.float32 if x_fp32 else torch.bfloat16
    dx = torch.empty((n, c, h, w), device=dev, dtype=dt, memory_format=torch.channels_last)
    with torch.cuda.device(dev):
        _lib.call("fp8_resample_down2_bwd", _ptr(dy), _ptr(dx), _DT[dt], n, h, w, c, _stream(dev))
    return dx


@resample_down2_bwd.register_fake
def _(dy, h, w, x_fp32):
    dt = torch.float32 if x_fp32 else torch.bfloat16
    return dy.new_empty((dy.shape[0], dy.shape[1], h, w), dtype=dt).contiguous(memory_format=torch.channels_last)


@torch.library.custom_op("fp8_b200::up_cat", mutates_args=())
def up_cat(a: torch.Tensor, s: torch.Tensor, factor: int, out_fp32: bool) -> torch.Tensor:
    """cat([upsample_nearest(a, factor), s], dim=1) in one pass (unet.py:379-383); fp32 or bf16 out."""
    dev = _require_cuda(a, s)
    _resample_check(a, "a")
    _resample_check(s, "s")
    n, c1, ha, wa = a.shape
    c2, h, w = s.shape[1], s.shape[2], s.shape[3]
    if (s.shape[0], h, w) != (n, ha * factor, wa * factor):
        raise RuntimeError("a upsampled by factor must match s in batch and spatial size")
    dt = torch.float32 if out_fp32 else torch.bfloat16
    y = torch.empty((n, c1 + c2, h, w), device=dev, dtype=dt, memory_format=torch.channels_last)
    with torch.cuda.device(dev):
        _lib.call("fp8_up_cat", _ptr(a), _DT[a.dtype], _ptr(s), _DT[s.dtype], _ptr(y), _DT[dt], n, h, w, c1, c2,
                  factor, _stream(dev))
    return y


@up_cat.register_fake
def _(a, s, factor, out_fp32):
    dt = torch.float32 if out_fp32 else torch.bfloat16
    return a.new_empty((a.shape[0], a.shape[1] + s.shape[1], s.shape[2], s.shape[3]), dtype=dt).contiguous(
        memory_format=torch.channels_last)


@torch.library.custom_op("fp8_b200::up_cat_bwd", mutates_args=())
def up_cat_bwd(dy: torch.Tensor, c1: int, factor: int, a_fp32: bool,
               s_fp32: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Gradients of up_cat: (block sums of dy[:, :c1] in a's dtype, dy[:, c1:] in s's dtype)."""
    dev = _require_cuda(dy)
    dy = dy.contiguous(memory_format=torch.channels_last)
    _resample_check(dy, "dy")
    n, c, h, w = dy.shape
    ta = torch.float32 if a_fp32 else torch.bfloat16
    ts = torch.float32 if s_fp32 else torch.bfloat16
    da = torch.empty((n, c1, h // factor, w // factor), device=dev, dtype=ta, memory_format=torch.channels_last)
    ds = torch.empty((n, c - c1, h, w), device=dev, dtype=ts, memory_format=torch.channels_last)
    with torch.cuda.device(dev):
        _lib.call("fp8_up_cat_bwd", _ptr(dy), _DT[dy.dtype], _ptr(da), _DT[ta], _ptr(ds), _DT[ts], n, h, w, c1,
                  c - c1, factor, _stream(dev))
    return da, ds


@up_cat_bwd.register_fake
def _(dy, c1, factor, a_fp32, s_fp32):
    n, c, h, w = dy.shape
    ta = torch.float32 if a_fp32 else torch.bfloat16
    ts = torch.float32 if s_fp32 else torch.bfloat16
    cl = torch.channels_last
    return (dy.new_empty((n, c1, h // factor, w // factor), dtype=ta).contiguous(memory_format=cl),
            dy.new_empty((n, c - c1, h, w), dtype=ts).contiguous(memory_format=cl))


@torch.library.custom_op("fp8_b200::up_cat_pair", mutates_args=())
def up_cat_pair(a: torch.Tensor, s: torch.Tensor, factor: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(y, bf16(y)) for the fp32 y of up_cat: the concatenation and the copy bf16 autocast
    makes of it for the next block's 1x1 skip conv (unet.py:139, 161), in one pass."""
    dev = _require_cuda(a, s)
    _resample_check(a, "a")
    _resample_check(s, "s")
    n, c1, ha, wa = a.shape
    c2, h, w = s.shape[1], s.shape[2], s.shape[3]
    if (s.shape[0], h, w) != (n, ha * factor, wa * factor):
        raise RuntimeError("a upsampled by factor must match s in batch and spatial size")
    y = torch.empty((n, c1 + c2, h, w), device=dev, dtype=torch.float32, memory_format=torch.channels_last)
    y16 = torch.empty((n, c1 + c2, h, w), device=dev, dtype=torch.bfloat16, memory_format=torch.channels_last)
    with torch.cuda.device(dev):
        _lib.call("fp8_up_cat_pair", _ptr(a), _DT[a.dtype], _ptr(s), _DT[s.dtype], _ptr(y), _ptr(y16), n, h, w, c1,
                  c2, factor, _stream(dev))
    return y, y16


@up_cat_pair.register_fake
def _(a, s, factor):
    shape = (a.shape[0], a.shape[1] + s.shape[1], s.shape[2], s.shape[3])
    cl = torch.channels_last
    return (a.new_empty(shape, dtype=torch.float32).contiguous(memory_format=cl),
            a.new_empty(shape, dtype=torch.bfloat16).contiguous(memory_format=cl))


@torch.library.custom_op("fp8_b200::up_cat_pair_bwd", mutates_args=())
def up_cat_pair_bwd(dy: torch.Tensor, dy16: torch.Tensor, c1: int, factor: int, a_fp32: bool,
                    s_fp32: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Gradients of up_cat_pair: up_cat_bwd of dy + dy16 (summed in fp32, as autograd sums them)."""
    dev = _require_cuda(dy, dy16)
    dy = dy.contiguous(memory_format=torch.channels_last)
    dy16 = dy16.contiguous(memory_format=torch.channels_last)
    _resample_check(dy, "dy")
    _resample_check(dy16, "dy16")
    if dy.dtype != torch.float32 or dy16.dtype != torch.bfloat16 or dy.shape != dy16.shape:
        raise RuntimeError("dy must be float32 and dy16 bfloat16 of one shape")
    n, c, h, w = dy.shape
    ta = torch.float32 if a_fp32 else torch.bfloat16
    ts = torch.float32 if s_fp32 else torch.bfloat16
    da = torch.empty((n, c1, h // factor, w // factor), device=dev, dtype=ta, memory_format=torch.channels_last)
    ds = torch.empty((n, c - c1, h, w), device=dev, dtype=ts, memory_format=torch.channels_last)
    with torch.cuda.device(dev):
        _lib.call("fp8_up_cat_pair_bwd", _ptr(dy), _ptr(dy16), _ptr(da), _DT[ta], _ptr(ds), _DT[ts], n, h, w, c1,
                  c - c1, factor, _stream(dev))
    return da, ds


@up_cat_pair_bwd.register_fake
def _(dy, dy16, c1, factor, a_fp32, s_fp32):
    n, c, h, w = dy.shape
    ta = torch.float32 if a_fp32 else torch.bfloat16
    ts = torch.float32 if s_fp32 else torch.bfloat16
    cl = torch.channels_last
    return (dy.new_empty((n, c1, h // factor, w // factor), dtype=ta).contiguous(memory_format=cl),
            dy.new_empty((n, c - c1, h, w), dtype=ts).contiguous(memory_format=cl))


@torch.library.custom_op("fp8_b200::add_scale", mutates_args=())
def add_scale(a: torch.Tensor, b: torch.Tensor, inv: float) -> torch.Tensor:
    """RN(RN(a + b) * inv) in the wider dtype of a and b (same shape and dense layout)."""
    dev = _require_cuda(a, b)
    dt = torch.promote_types(a.dtype, b.dtype)
    y = torch.empty_like(a, dtype=dt)
    with torch.cuda.device(dev):
        _lib.call("fp8_add_scale", _ptr(a), _DT[a.dtype], _ptr(b), _DT[b.dtype], _ptr(y), _DT[dt], a.numel(),
                  float(inv), _stream(dev))
    return y


@add_scale.register_fake
def _(a, b, inv):
    return torch.empty_like(a, dtype=torch.promote_types(a.dtype, b.dtype))


@torch.library.custom_op("fp8_b200::add_scale_bwd", mutates_args=())
def add_scale_bwd(dy: torch.Tensor, inv: float, a_fp32: bool, b_fp32: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """Gradients of add_scale: RN(dy * inv) in each input's dtype."""
    dev = _require_cuda(dy)
    if dy.dtype not in _DT or not (dy.is_contiguous() or (dy.dim() == 4 and dy.is_contiguous(
            memory_format=torch.channels_last))):
        dy = dy.contiguous(memory_format=torch.channels_last) if dy.dim() == 4 else dy.contiguous()
    da = torch.empty_like(dy, dtype=torch.float32 if a_fp32 else torch.bfloat16)
    db = torch.empty_like(dy, dtype=torch.float32 if b_fp32 else torch.bfloat16)
    with torch.cuda.device(dev):
        _lib.call("fp8_add_scale_bwd", _ptr(dy), _DT[dy.dtype], _ptr(da), _DT[da.dtype], _ptr(db), _DT[db.dtype],
                  dy.numel(), float(inv), _stream(dev))
    return da, db


@add_scale_bwd.register_fake
def _(dy, inv, a_fp32, b_fp32):
    return (torch.empty_like(dy, dtype=torch.float32 if a_fp32 else torch.bfloat16),
            torch.empty_like(dy, dtype=torch.float32 if b_fp32 else torch.bfloat16))


@torch.library.custom_op("fp8_b200::add_scale_bwd_quant", mutates_args=("window",))
def add_scale_bwd_quant(dy: torch.Tensor, inv: float, a_fp32: bool, window: torch.Tensor,
                        pos: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """add_scale_bwd with b bf16, plus db's delayed e4m3 cast -> (da, db, dbq, scale used).

    dbq and the scale used are those of ``quantize_delayed_window(db, window, pos, False)`` (the
    backward quantize of the FP8 conv whose output is b), and db's own scale lands at
    ``window[pos]`` as there; db is not read again."""
    dev = _require_cuda(dy, window, pos)
    _check_window(window, pos, dev)
    if dy.dim() != 4 or dy.dtype not in _DT:
        raise RuntimeError("add_scale_bwd_quant expects a 4-D bfloat16 / float32 gradient")
    dy = dy.contiguous(memory_format=torch.channels_last)
    da = torch.empty_like(dy, dtype=torch.float32 if a_fp32 else torch.bfloat16)
    db = torch.empty_like(dy, dtype=torch.bfloat16)
    dbq = torch.empty_like(dy, dtype=FP8_DTYPE)
    used = torch.empty((), device=dev, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(max(lib.fp8_add_scale_bwd_quant_workspace_bytes(dy.numel()) // 4, 1), device=dev,
                         dtype=torch.float32)
        _lib.call("fp8_add_scale_bwd_quant", _ptr(dy), _DT[dy.dtype], _ptr(da), _DT[da.dtype], _ptr(db), _ptr(dbq),
                  _ptr(window), window.numel(), _ptr(pos), _ptr(used), dy.numel(), float(inv), _ptr(ws),
                  ws.numel() * 4, _stream(dev))
    return da, db, dbq, used


@add_scale_bwd_quant.register_fake
def _(dy, inv, a_fp32, window, pos):
    cl = torch.channels_last
    return (torch.empty_like(dy, dtype=torch.float32 if a_fp32 else torch.bfloat16, memory_format=cl),
            torch.empty_like(dy, dtype=torch.bfloat16, memory_format=cl),
            torch.empty_like(dy, dtype=FP8_DTYPE, memory_format=cl), dy.new_empty((), dtype=torch.float32))


@torch.library.custom_op("fp8_b200::gn_act_quant_fwd", mutates_args=())
def gn_act_quant_fwd(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, film: torch.Tensor | None,
                     seed: torch.Tensor | None, prev_scale: torch.Tensor, p: float, eps: float,
                     groups: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """gn_act_fwd fused with quantize_fp8_delayed of its output -> (e4m3 channels_last, current scale, stats).

    The e4m3 bytes and the scale are bit for bit those of
    ``quantize_fp8_delayed(gn_act_fwd(...)[0], prev_scale)`` (fp8_kernels.py:518-556);
    the bf16 activation itself is never written."""
    dev = _require_cuda(x, gamma, beta)
    n, c, hw = _gn_check(x, gamma, beta, film, groups)
    _check_scale(prev_scale, dev, "prev_scale")
    q = torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.channels_last)
    scale = torch.empty((), device=dev, dtype=torch.float32)
    stats = torch.empty((n, 2, groups), device=dev, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(max(lib.fp8_gn_act_quant_workspace_bytes(n, hw, c) // 4, 4), device=dev,
                         dtype=torch.float32)
        _lib.check(lib.fp8_gn_act_quant_fwd(
            _ptr(x), int(x.dtype == torch.float32), _ptr(gamma), _ptr(beta), _ptr(film), _film_ld(film, c), _ptr(seed),
            float(p), float(eps), _ptr(prev_scale), _ptr(stats), _ptr(q), _ptr(scale), n, hw, c, groups, _ptr(ws),
            ws.numel() * 4, _stream(dev)), "fp8_gn_act_quant_fwd")
    return q, scale, stats


@torch.library.custom_op("fp8_b200::gn_act_quant_fwd_window", mutates_args=("window", "pos"))
def gn_act_quant_fwd_window(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, film: torch.Tensor | None,
                            seed: torch.Tensor | None, window: torch.Tensor, pos: torch.Tensor, advance: bool,
                            p: float, eps: float, groups: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """gn_act_quant_fwd with the scale history on the device -> (e4m3, scale used, stats)."""
    dev = _require_cuda(x, gamma, beta)
    n, c, hw = _gn_check(x, gamma, beta, film, groups)
    _check_window(window, pos, dev)
    q = torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.channels_last)
    used = torch.empty((), device=dev, dtype=torch.float32)
    stats = torch.empty((n, 2, groups), device=dev, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(max(lib.fp8_gn_act_quant_workspace_bytes(n, hw, c) // 4, 4), device=dev,
                         dtype=torch.float32)
        _lib.check(lib.fp8_gn_act_quant_fwd_window(
            _ptr(x), int(x.dtype == torch.float32), _ptr(gamma), _ptr(beta), _ptr(film), _film_ld(film, c), _ptr(seed),
            float(p), float(eps), _ptr(window), window.numel(), _ptr(pos), int(advance), _ptr(used), _ptr(stats),
            _ptr(q), n, hw, c, groups, _ptr(ws), ws.numel() * 4, _stream(dev)), "fp8_gn_act_quant_fwd_window")
    return q, used, stats


@gn_act_quant_fwd_window.register_fake
def _(x, gamma, beta, film, seed, window, pos, advance, p, eps, groups):
    return (torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.channels_last),
            x.new_empty((), dtype=torch.float32), x.new_empty((x.shape[0], 2, groups), dtype=torch.float32))


@gn_act_quant_fwd.register_fake
def _(x, gamma, beta, film, seed, prev_scale, p, eps, groups):
    return (torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.channels_last),
            x.new_empty((), dtype=torch.float32), x.new_empty((x.shape[0], 2, groups), dtype=torch.float32))


@torch.library.custom_op("fp8_b200::gn_act_bwd", mutates_args=())
def gn_act_bwd(x: torch.Tensor, dy: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
               film: torch.Tensor | None, seed: torch.Tensor | None, stats: torch.Tensor, p: float, eps: float,
               groups: int, dx_add: torch.Tensor | None = None
               ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Backward of gn_act_fwd -> (dx in x's dtype, channels_last; dgamma, dbeta fp32 [C]; dfilm bf16 [N, 2C], or
    an empty tensor without FiLM).  ``dx_add``: a second gradient of x (x's dtype and shape), added to dx as
    autograd would sum the two."""
    dev = _require_cuda(x, dy, gamma, beta, stats)
    n, c, hw = _gn_check(x, gamma, beta, film, groups)
    dy = dy.contiguous(memory_format=torch.channels_last)
    if dy.dtype != torch.bfloat16 or dy.shape != x.shape:
        raise RuntimeError("dy must be a bfloat16 tensor shaped like x")
    if dx_add is not None:
        dx_add = dx_add.contiguous(memory_format=torch.channels_last)
        if dx_add.dtype != x.dtype or dx_add.shape != x.shape or dx_add.device != dev:
            raise RuntimeError("dx_add must have x's dtype, shape and device")
    dx = torch.empty_like(x, memory_format=torch.channels_last)
    totals = torch.empty((n, 3, c), device=dev, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(max(lib.fp8_gn_workspace_bytes(n, hw, c) // 4, 4), device=dev, dtype=torch.float32)
        common = (_ptr(x), int(x.dtype == torch.float32), _ptr(dy), _ptr(gamma), _ptr(beta), _ptr(film),
                  _film_ld(film, c), _ptr(seed), float(p), float(eps), _ptr(stats), _ptr(totals))
        tail = (n, hw, c, groups, _ptr(ws), ws.numel() * 4, _stream(dev))
        if dx_add is None:
            _lib.check(lib.fp8_gn_act_bwd(*common, _ptr(dx), *tail), "fp8_gn_act_bwd")
        else:
            _lib.check(lib.fp8_gn_act_bwd_accumulate(*common, _ptr(dx_add), _ptr(dx), *tail),
                       "fp8_gn_act_bwd_accumulate")
        dgamma = torch.empty((c,), device=dev, dtype=torch.float32)
        dbeta = torch.empty((c,), device=dev, dtype=torch.float32)
        dfilm = torch.empty((n, 2 * c) if film is not None else (0,), device=dev, dtype=torch.bfloat16)
        _lib.check(lib.fp8_gn_param_grads(_ptr(totals), _ptr(film), _film_ld(film, c), n, c, _ptr(dgamma), _ptr(dbeta),
                                          _ptr(dfilm) if film is not None else None, 2 * c, _stream(dev)),
                   "fp8_gn_param_grads")
    return dx, dgamma, dbeta, dfilm


@torch.library.custom_op("fp8_b200::gn_act_bwd_quant", mutates_args=("window",))
def gn_act_bwd_quant(x: torch.Tensor, dy: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor,
                     film: torch.Tensor | None, seed: torch.Tensor | None, stats: torch.Tensor, p: float, eps: float,
                     groups: int, window: torch.Tensor, pos: torch.Tensor
                     ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """gn_act_bwd for a bf16 x, plus dx's delayed e4m3 cast -> (dx, dgamma, dbeta, dfilm, dxq, scale used).

    dxq and the scale used are those of ``quantize_delayed_window(dx, window, pos, False)`` (the backward
    quantize of the FP8 conv whose output is x), and dx's own scale lands at ``window[pos]``."""
    dev = _require_cuda(x, dy, gamma, beta, stats, window, pos)
    n, c, hw = _gn_check(x, gamma, beta, film, groups)
    _check_window(window, pos, dev)
    if x.dtype != torch.bfloat16:
        raise RuntimeError("gn_act_bwd_quant expects a bfloat16 x")
    dy = dy.contiguous(memory_format=torch.channels_last)
    if dy.dtype != torch.bfloat16 or dy.shape != x.shape:
        raise RuntimeError("dy must be a bfloat16 tensor shaped like x")
    dx = torch.empty_like(x, memory_format=torch.channels_last)
    dxq = torch.empty_like(x, dtype=FP8_DTYPE, memory_format=torch.channels_last)
    used = torch.empty((), device=dev, dtype=torch.float32)
    totals = torch.empty((n, 3, c), device=dev, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(dev):
        ws = torch.empty(max(lib.fp8_gn_act_bwd_quant_workspace_bytes(n, hw, c) // 4, 4), device=dev,
                         dtype=torch.float32)
        _lib.check(lib.fp8_gn_act_bwd_quant(
            _ptr(x), _ptr(dy), _ptr(gamma), _ptr(beta), _ptr(film), _film_ld(film, c), _ptr(seed), float(p),
            float(eps), _ptr(stats), _ptr(totals), _ptr(dx), _ptr(dxq), _ptr(window), window.numel(), _ptr(pos),
            _ptr(used), n, hw, c, groups, _ptr(ws), ws.numel() * 4, _stream(dev)), "fp8_gn_act_bwd_quant")
        dgamma = torch.empty((c,), device=dev, dtype=torch.float32)
        dbeta = torch.empty((c,), device=dev, dtype=torch.float32)
        dfilm = torch.empty((n, 2 * c) if film is not None else (0,), device=dev, dtype=torch.bfloat16)
        _lib.check(lib.fp8_gn_param_grads(_ptr(totals), _ptr(film), _film_ld(film, c), n, c, _ptr(dgamma), _ptr(dbeta),
                                          _ptr(dfilm) if film is not None else None, 2 * c, _stream(dev)),
                   "fp8_gn_param_grads")
    return dx, dgamma, dbeta, dfilm, dxq, used


@gn_act_bwd_quant.register_fake
def _(x, dy, gamma, beta, film, seed, stats, p, eps, groups, window, pos):
    n, c = x.shape[0], x.shape[1]
    cl = torch.channels_last
    return (torch.empty_like(x, memory_format=cl), x.new_empty((c,), dtype=torch.float32),
            x.new_empty((c,), dtype=torch.float32),
            x.new_empty((n, 2 * c) if film is not None else (0,), dtype=torch.bfloat16),
            torch.empty_like(x, dtype=FP8_DTYPE, memory_format=cl), x.new_empty((), dtype=torch.float32))


@gn_act_bwd.register_fake
def _(x, dy, gamma, beta, film, seed, stats, p, eps, groups, dx_add=None):
    n, c = x.shape[0], x.shape[1]
    return (torch.empty_like(x, memory_format=torch.channels_last), x.new_empty((c,), dtype=torch.float32),
            x.new_empty((c,), dtype=torch.float32),
            x.new_empty((n, 2 * c) if film is not None else (0,), dtype=torch.bfloat16))
