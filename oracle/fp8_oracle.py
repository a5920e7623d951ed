"""CPU oracle for the FP8 hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this module, and only as the checker (or as the timed
CPU restatement of the reference).  The product path (``fp8_b200``) never calls
it and has no CPU fallback.

It restates the reference's arithmetic (fattorib/diffusion-profiled,
diffusion/fp8_kernels.py) on the CPU:

* quantize (current scaling, :54-64 + :90-102 + :105-120 via :559-601):
    amax = max|x| (fp32), s = amax/448 if amax > 0 else 1 (fp32 IEEE divide),
    q = e4m3(max(-448, min(x/s, 448)))  — min/max ignore NaN like Triton's
    tl.minimum/tl.maximum default, so 0/0 maps to +448.
* quantize (delayed scaling, :69-87 via :518-556): cast with the previous scale,
  report the scale of the tensor's own amax.
* conv fwd / dX / dW (:168-247, :250-318, :385-468) and the new FP8 linear:
  fp32-accumulating torch CPU conv / matmul on the dequantised operands, times
  the product of the two scales, rounded to bf16 (the reference multiplies the
  fp32 accumulator by ``sa*sb`` and stores bf16).

The e4m3 encoder below is written from the format definition (1 sign bit, 4
exponent bits with bias 7, 3 mantissa bits, no infinities, 0x7F/0xFF = NaN,
max finite 448, round to nearest even, subnormal step 2**-9); the tests pin it
against torch's ``float8_e4m3fn`` conversion exhaustively.

Parity anchor: the reference has no tests or golden vectors of its own.  The
conv index conventions are pinned against the reference's own Triton kernels run
under the Triton CPU interpreter (tests/golden/make_golden.py → fixtures); the
byte-level cast is pinned against torch's e4m3fn conversion, because the Triton
interpreter's fp32→fp8 store mis-rounds (on config 1's X, 66,045 of 2,097,152
bytes differ from torch's conversion, e.g. 31.63 → 16 where torch gives 32).
"""

from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

E4M3_MAX = 448.0


# ----------------------------------------------------------------------------- e4m3 format
def e4m3_encode(v: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even, saturating (|v| > 448 -> 448) encode of float values to e4m3fn bytes.

    NaN inputs encode to 0x7F (sign kept).  Works elementwise on any shape.
    """
    v = np.asarray(v, dtype=np.float64)
    sign = np.signbit(v).astype(np.uint8) << 7
    a = np.abs(v)
    nan = np.isnan(a)
    a = np.where(nan, 0.0, np.minimum(a, E4M3_MAX))
    out = np.zeros(a.shape, dtype=np.uint8)

    normal = a >= 2.0**-6
    # normal numbers: a = 2**e * (1 + m/8)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(normal, a, 1.0))).astype(np.int64)
    # guard against log2 rounding at exact powers of two
    e = np.where(normal & (np.ldexp(1.0, e) > a), e - 1, e)
    e = np.where(normal & (np.ldexp(1.0, e + 1) <= a), e + 1, e)
    r = np.rint(np.ldexp(a, -(e - 3)))  # in [8, 16]; np.rint is round-half-even
    carry = r >= 16
    r = np.where(carry, 8, r)
    e = np.where(carry, e + 1, e)
    nbyte = ((e + 7) << 3) | (r.astype(np.int64) - 8)
    # subnormals (and zero): multiples of 2**-9
    rs = np.rint(np.ldexp(a, 9)).astype(np.int64)  # 0..8 (8 == smallest normal, same byte 0x08)
    out = np.where(normal, nbyte, rs).astype(np.uint8)
    out = np.where(nan, np.uint8(0x7F), out)
    return (out | sign).astype(np.uint8)


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    """e4m3fn bytes -> float32 values (NaN for 0x7F / 0xFF)."""
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, np.ldexp(m.astype(np.float64), -9), np.ldexp(1.0 + m / 8.0, e - 7))
    val = np.where((e == 0xF) & (m == 0x7), np.nan, val)
    return (s * val).astype(np.float32)


# ----------------------------------------------------------------------------- quantize
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _as_f32(x) -> np.ndarray:
    """bf16 torch tensor (any layout) -> float32 numpy array in *memory* order."""
    if isinstance(x, torch.Tensor):
        t = x.detach().cpu()
        if t.dtype == torch.bfloat16:
            # memory order: the reference quantizes the flat buffer (fp8_kernels.py:61, :116)
            flat = t.as_strided((t.numel(),), (1,)) if _is_dense(t) else t.reshape(-1)
            return bf16_bits_to_f32(flat.contiguous().view(torch.int16).numpy().view(np.uint16))
        return t.reshape(-1).float().numpy()
    return np.asarray(x, dtype=np.float32).reshape(-1)


def _is_dense(t: torch.Tensor) -> bool:
    return t.is_contiguous() or (t.dim() == 4 and t.is_contiguous(memory_format=torch.channels_last))


def amax_scale(vals_f32: np.ndarray) -> np.float32:
    """finalize_amax_kernel (fp8_kernels.py:90-102): amax/448 in fp32, or 1.0 for amax == 0.
    The amax ignores NaN: the reference's tl.max (fp8_kernels.py:62, :98) reduces with the
    GPU's max.f32, which returns the other operand when one is NaN (np.fmax); a tensor that
    is all NaN gets scale 1.0 either way."""
    a = np.float32(np.fmax.reduce(np.abs(vals_f32).ravel())) if vals_f32.size else np.float32(0.0)
    return np.float32(a / np.float32(E4M3_MAX)) if a > 0 else np.float32(1.0)


def cast_with_scale(vals_f32: np.ndarray, scale: np.float32) -> np.ndarray:
    """quantize_fp8_kernel body (fp8_kernels.py:116-120): fp32 divide, min then max, e4m3 cast."""
    with np.errstate(divide="ignore", invalid="ignore"):
        t = vals_f32.astype(np.float32) / np.float32(scale)
    t = np.fmin(t, np.float32(E4M3_MAX))
    t = np.fmax(np.float32(-E4M3_MAX), t)
    return e4m3_encode(t)


def quantize_current(x) -> tuple[np.ndarray, np.float32]:
    """quantize_fp8 (fp8_kernels.py:559-601) -> (e4m3 bytes in memory order, scale)."""
    v = _as_f32(x)
    s = amax_scale(v)
    return cast_with_scale(v, s), s


def quantize_delayed(x, prev_scale: float) -> tuple[np.ndarray, np.float32]:
    """quantize_fp8_delayed (fp8_kernels.py:518-556) -> (bytes cast with prev_scale, own scale)."""
    v = _as_f32(x)
    return cast_with_scale(v, np.float32(prev_scale)), amax_scale(v)


def bytes_like(q: np.ndarray, like: torch.Tensor) -> torch.Tensor:
    """Wrap memory-order e4m3 bytes into a float8 tensor with ``like``'s shape and strides."""
    flat = torch.from_numpy(np.ascontiguousarray(q)).view(torch.float8_e4m3fn)
    out = torch.empty_like(like, dtype=torch.float8_e4m3fn, device="cpu", memory_format=torch.preserve_format)
    out.as_strided((out.numel(),), (1,)).copy_(flat)
    return out


def quantize_tensor(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Torch-facing current-scaling oracle: (float8 tensor like x, 0-d fp32 scale)."""
    q, s = quantize_current(x)
    return bytes_like(q, x), torch.tensor(s, dtype=torch.float32)


# ----------------------------------------------------------------------------- contractions
def _f32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().cpu().float()


def _finish(acc: torch.Tensor, scale: float, bias=None, silu: bool = False, f32: bool = False) -> torch.Tensor:
    """Epilogue: ``acc * scale (+ bias) (silu)`` in fp32, then round-to-nearest-even to bf16.

    ``f32=True`` returns the fp32 value before the final rounding.
    """
    y = acc * torch.tensor(np.float32(scale), dtype=torch.float32)
    if bias is not None:
        b = _f32(bias)
        y = y + (b.view(1, -1, 1, 1) if y.dim() == 4 else b.view(1, -1))
    if silu:
        y = F.silu(y)
    return y if f32 else y.to(torch.bfloat16)


def round_bf16_toward_zero(y: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 by truncation (the rounding of the Triton CPU interpreter's bf16 stores)."""
    bits = y.detach().cpu().float().contiguous().view(torch.int32) & ~0xFFFF
    return bits.view(torch.float32).to(torch.bfloat16)


def conv_fwd(xq, wq, sx, sw, bias=None, silu: bool = False, f32: bool = False) -> torch.Tensor:
    """conv2d_fwd_fp8_kernel (fp8_kernels.py:168-247): bf16 ``conv(xq, wq, pad=1) * (sx*sw)``."""
    acc = F.conv2d(_f32(xq), _f32(wq), padding=1)
    scale = np.float32(np.float32(sx) * np.float32(sw))
    return _finish(acc, scale, bias, silu, f32).contiguous(memory_format=torch.channels_last)


def conv_dx(dyq, wq, sdy, sw, f32: bool = False) -> torch.Tensor:
    """conv2d_dx_fp8_kernel (fp8_kernels.py:250-318): bf16 input gradient."""
    dy = _f32(dyq)
    w = _f32(wq)
    acc = torch.nn.grad.conv2d_input((dy.shape[0], w.shape[1], dy.shape[2], dy.shape[3]), w, dy, padding=1)
    scale = np.float32(np.float32(sdy) * np.float32(sw))
    return _finish(acc, scale, f32=f32).contiguous(memory_format=torch.channels_last)


def conv_dw(xq, dyq, sx, sdy, f32: bool = False) -> torch.Tensor:
    """conv2d_dw_fp8_kernel + reduce (fp8_kernels.py:385-468): bf16 weight gradient."""
    x = _f32(xq)
    dy = _f32(dyq)
    acc = torch.nn.grad.conv2d_weight(x, (dy.shape[1], x.shape[1], 3, 3), dy, padding=1)
    scale = np.float32(np.float32(sx) * np.float32(sdy))
    return _finish(acc, scale, f32=f32).contiguous(memory_format=torch.channels_last)


def linear_fwd(xq, wq, sx, sw, bias=None, silu: bool = False) -> torch.Tensor:
    """New FP8 linear: bf16 ``(xq @ wq.T) * (sx*sw) (+ b)``; wq in nn.Linear [out, in] layout."""
    acc = _f32(xq) @ _f32(wq).T
    scale = np.float32(np.float32(sx) * np.float32(sw))
    return _finish(acc, scale, bias, silu)


def linear_dx(dyq, wq, sdy, sw) -> torch.Tensor:
    acc = _f32(dyq) @ _f32(wq)
    return _finish(acc, np.float32(np.float32(sdy) * np.float32(sw)))


def linear_dw(dyq, xq, sdy, sx) -> torch.Tensor:
    acc = _f32(dyq).T @ _f32(xq)
    return _finish(acc, np.float32(np.float32(sdy) * np.float32(sx)))


# ----------------------------------------------------------------------------- attention
def _e4m3_values(x: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """The attention kernels' cast: e4m3 grid values of RN(x * r), r = RN(1 / scale) in fp32,
    saturating at +-448, round to nearest even."""
    r = (np.float32(1.0) / scale.astype(np.float32)).astype(np.float32)
    t = (x.astype(np.float32) * r).astype(np.float32)
    t = np.fmax(np.float32(-E4M3_MAX), np.fmin(t, np.float32(E4M3_MAX)))
    return e4m3_decode(e4m3_encode(t))


def _split_heads(qkv: torch.Tensor, heads: int) -> np.ndarray:
    b, seq, c3 = qkv.shape
    x = qkv.detach().cpu().float().numpy().reshape(b, seq, 3, heads, c3 // (3 * heads))
    return x.transpose(2, 0, 3, 1, 4)  # [3, B, heads, L, 64]


def attention_quantized(qkv: torch.Tensor, heads: int):
    """Per (image, head): the e4m3 values of q, k, v and their scales amax/448 (1 if amax is 0;
    the reference's per-tensor scale, fp8_kernels.py:90-102, of each head slice), cast as
    e4m3(x * (1/s))."""
    x = _split_heads(qkv, heads)
    amax = np.abs(x).max(axis=(3, 4)).astype(np.float32)  # [3, B, heads]
    with np.errstate(divide="ignore", invalid="ignore"):
        scale = np.where(amax > 0, amax / np.float32(E4M3_MAX), np.float32(1.0)).astype(np.float32)
    vals = _e4m3_values(x, scale[..., None, None])
    return vals, scale


def attention_fwd(qkv: torch.Tensor, heads: int):
    """FP8 attention forward as attn_fwd_fp8_kernel computes it -> (o bf16 [B, L, C], lse [B, heads, L],
    scales [B, heads, 3]): S = q k^T (e4m3 values), p = exp((S - max) * sq sk / 8), l = sum p,
    o = (e4m3(p * 448) v) * sv / (448 l)."""
    vals, scale = attention_quantized(qkv, heads)
    q, k, v = (vals[i].astype(np.float64) for i in range(3))
    sv = scale[2].astype(np.float64)[..., None, None]
    c = (np.float32(scale[0]) * np.float32(scale[1]) * np.float32(0.125)).astype(np.float64)[..., None, None]
    s = q @ k.transpose(0, 1, 3, 2)
    m = s.max(axis=-1, keepdims=True)
    p = np.exp((s - m) * c)
    l = p.sum(axis=-1, keepdims=True)
    pq = e4m3_decode(e4m3_encode((p * 448.0).astype(np.float32))).astype(np.float64)
    o = (pq @ v) * sv / (448.0 * l)  # [B, heads, L, 64]
    b, h, seq, d = o.shape
    o_t = torch.from_numpy(o.transpose(0, 2, 1, 3).reshape(b, seq, h * d).astype(np.float32)).to(torch.bfloat16)
    lse = torch.from_numpy((m * c + np.log(l))[..., 0].astype(np.float32))
    return o_t, lse, torch.from_numpy(scale.transpose(1, 2, 0).copy())


def attention_bwd(qkv: torch.Tensor, o: torch.Tensor, do: torch.Tensor, lse: torch.Tensor, heads: int) -> torch.Tensor:
    """attn_bwd_kernel's gradient -> d(qkv) bf16: P = exp(S c - lse), dP = sv dO v^T,
    dS = P (dP - rowsum(dO o O)); P and dS rounded to bf16; dV = P^T dO, dK = sq/8 dS^T q,
    dQ = sk/8 dS k (q, k, v their e4m3 values)."""
    vals, scale = attention_quantized(qkv, heads)
    q, k, v = (vals[i].astype(np.float64) for i in range(3))
    b, seq, c = o.shape
    d = c // heads
    split = lambda t: t.detach().cpu().float().numpy().reshape(b, seq, heads, d).transpose(0, 2, 1, 3)  # noqa: E731
    o_h, do_h = split(o).astype(np.float64), split(do).astype(np.float64)
    cs = (np.float32(scale[0]) * np.float32(scale[1]) * np.float32(0.125)).astype(np.float64)[..., None, None]
    sv = scale[2].astype(np.float64)[..., None, None]
    s = q @ k.transpose(0, 1, 3, 2)
    p = np.exp(s * cs - lse.detach().cpu().double().numpy()[..., None])
    dp = (do_h @ v.transpose(0, 1, 3, 2)) * sv
    delta = (do_h * o_h).sum(axis=-1, keepdims=True)
    ds = p * (dp - delta)
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16).float().double().numpy()  # noqa: E731
    p_b, ds_b = bf(p), bf(ds)
    dv = p_b.transpose(0, 1, 3, 2) @ do_h
    dk = (np.float32(0.125) * scale[0]).astype(np.float64)[..., None, None] * (ds_b.transpose(0, 1, 3, 2) @ q)
    dq = (np.float32(0.125) * scale[1]).astype(np.float64)[..., None, None] * (ds_b @ k)
    grads = np.stack([dq, dk, dv])  # [3, B, heads, L, d]
    out = grads.transpose(1, 3, 0, 2, 4).reshape(b, seq, 3 * c)
    return torch.from_numpy(out.astype(np.float32)).to(torch.bfloat16)


def attention_exact(qkv: torch.Tensor, heads: int) -> torch.Tensor:
    """Unquantized fp32 multi-head attention of the qkv projection output (the reference's
    scaled_dot_product_attention, unet.py:197) -> o fp32 [B, L, C]."""
    x = torch.from_numpy(_split_heads(qkv, heads).copy())
    o = F.scaled_dot_product_attention(x[0], x[1], x[2])
    b, h, seq, d = o.shape
    return o.transpose(1, 2).reshape(b, seq, h * d)


def max_rel_err(y: torch.Tensor, ref: torch.Tensor) -> float:
    """``max|y - ref| / max|ref|`` (the tolerance metric of the parity contract)."""
    y = y.detach().cpu().float()
    ref = ref.detach().cpu().float()
    denom = ref.abs().max().item()
    if denom == 0:
        return y.abs().max().item()
    return (y - ref).abs().max().item() / denom


__all__ = [
    "E4M3_MAX",
    "e4m3_encode",
    "e4m3_decode",
    "bf16_bits_to_f32",
    "amax_scale",
    "cast_with_scale",
    "quantize_current",
    "quantize_delayed",
    "bytes_like",
    "quantize_tensor",
    "conv_fwd",
    "conv_dx",
    "conv_dw",
    "linear_fwd",
    "linear_dx",
    "linear_dw",
    "max_rel_err",
    "round_bf16_toward_zero",
    "attention_quantized",
    "attention_fwd",
    "attention_bwd",
    "attention_exact",
]
