"""Generate the golden fixtures in this directory from the reference's own kernels.

Runs in the development container only (needs the reference checkout and
Triton's CPU interpreter); the fixtures it writes are committed so that the
tests never need the reference at run time.

    TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/reference

For each case it draws seeded inputs, quantises them with the oracle (the
reference's quantize semantics; see oracle/fp8_oracle.py), and runs the
reference Triton kernels from diffusion/fp8_kernels.py under the interpreter:

* partial_amax_kernel + finalize_amax_kernel (:54-64, :90-102)   -> current scale
* partial_amax_kernel_delayed + finalize_amax_kernel (:69-102)   -> delayed scale
* conv2d_fwd_fp8_kernel (:168-247, autotune bypassed with one of its configs)
* conv2d_dx_fp8_kernel (:250-318, with its DX_CONFIG_BY_SHAPE config)
* transpose_fp8_2d_kernel + conv2d_dw_fp8_kernel + conv2d_dw_reduce_fp8_kernel
  (:321-337, :385-468)

The fp8 bytes the interpreter stores are not used: its fp32->fp8 store
mis-rounds (e.g. 31.63 -> 16 where the e4m3 cast gives 32), so the byte-level
reference is the e4m3 cast itself (oracle encoder == torch float8_e4m3fn).
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "oracle"))
import fp8_oracle as oracle  # noqa: E402


def _bits_u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _bytes_u8(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.uint8).numpy().copy()


def _nhwc(t: torch.Tensor) -> torch.Tensor:
    """NCHW logical tensor -> physical NHWC contiguous copy."""
    return t.permute(0, 2, 3, 1).contiguous()


def gen_quantize_cases(fk) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(0)
    cases = {
        "randn": torch.randn(3, 5, 7, 11, generator=g),
        "zeros": torch.zeros(2, 3, 4, 5),
        "pow2": torch.randn(2, 4, 8, 8, generator=g).clamp(-1.9, 1.9).index_put_((torch.tensor([0]),) * 4,
                                                                                 torch.tensor(4.0)),
        "ragged": torch.randn(1, 1, 1, 8192 + 13, generator=g) * 37.0,
        "tiny": torch.randn(1, 2, 3, 5, generator=g) * 1e-3,
    }
    for name, x in cases.items():
        xb = x.to(torch.bfloat16).contiguous()
        n = xb.numel()
        n_part = (n + 8191) // 8192
        partials = torch.empty(n_part, dtype=torch.float32)
        scale = torch.empty((), dtype=torch.float32)
        fk.partial_amax_kernel[(n_part,)](xb, partials, n, BLOCK_SIZE=8192)
        block = 1 << max(0, (n_part - 1).bit_length())
        fk.finalize_amax_kernel[(1,)](partials, scale, n_partials=n_part, FP8_MAX_VALUE=fk.FP8_MAX_E4M3,
                                      BLOCK_SIZE=block)
        out[f"q_{name}_x"] = _bits_u16(xb)
        out[f"q_{name}_shape"] = np.array(xb.shape, dtype=np.int64)
        out[f"q_{name}_scale"] = np.array([scale.item()], dtype=np.float32)
        # delayed: previous scale 0.05 -> cast uses it, reported scale is the tensor's own
        prev = torch.tensor(0.05, dtype=torch.float32)
        qd = torch.empty(xb.shape, dtype=torch.float8_e4m3fn)
        partials2 = torch.empty(n_part, dtype=torch.float32)
        scale2 = torch.empty((), dtype=torch.float32)
        fk.partial_amax_kernel_delayed[(n_part,)](xb, qd, prev, partials2, n, FP8_MAX_VALUE=fk.FP8_MAX_E4M3,
                                                  BLOCK_SIZE=8192)
        fk.finalize_amax_kernel[(1,)](partials2, scale2, n_partials=n_part, FP8_MAX_VALUE=fk.FP8_MAX_E4M3,
                                      BLOCK_SIZE=block)
        out[f"q_{name}_delayed_prev"] = np.array([0.05], dtype=np.float32)
        out[f"q_{name}_delayed_scale"] = np.array([scale2.item()], dtype=np.float32)
    return out


def gen_conv_case(fk, tag: str, batch: int, cin: int, cout: int, h: int, w: int, seed: int) -> dict:
    import triton

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, cin, h, w, generator=g).to(torch.bfloat16)
    wt = (torch.rand(cout, cin, 3, 3, generator=g) * 2 - 1) / np.sqrt(cin * 9)
    wt = wt.to(torch.bfloat16)
    dy = (torch.randn(batch, cout, h, w, generator=g) * 1e-2).to(torch.bfloat16)

    x_cl = x.contiguous(memory_format=torch.channels_last)
    w_cl = wt.contiguous(memory_format=torch.channels_last)
    dy_cl = dy.contiguous(memory_format=torch.channels_last)
    xq, sx = oracle.quantize_tensor(x_cl)
    wq, sw = oracle.quantize_tensor(w_cl)
    dyq, sdy = oracle.quantize_tensor(dy_cl)

    # forward
    y = torch.empty(batch, cout, h, w, dtype=torch.bfloat16).contiguous(memory_format=torch.channels_last)
    m = batch * h * w
    grid = (triton.cdiv(m, 64), triton.cdiv(cout, 64))
    fk.conv2d_fwd_fp8_kernel.fn[grid](
        xq, wq, y, sx, sw, *xq.stride(), *wq.stride(), *y.stride(),
        BATCH=batch, IN_H=h, IN_W=w, CIN=cin, COUT=cout, BLOCK_M=64, BLOCK_N=64, BLOCK_K=32,
    )
    # data gradient (the reference's own per-shape launch config)
    dx = torch.empty(batch, cin, h, w, dtype=torch.bfloat16).contiguous(memory_format=torch.channels_last)
    grid = (triton.cdiv(cin, 64), triton.cdiv(m, 128))
    fk.conv2d_dx_fp8_kernel[grid](
        dyq, wq, dx, sdy, sw, *dyq.stride(), *wq.stride(), *dx.stride(),
        BATCH=batch, IN_H=h, IN_W=w, CIN=cin, COUT=cout, BLOCK_M=128, BLOCK_N=64, BLOCK_K=32,
    )
    # weight gradient: transpose dY, split-K GEMM, reduce
    split_k = 2
    dy_t = torch.empty((cout, m), dtype=dyq.dtype)
    fk.transpose_fp8_2d_kernel[(triton.cdiv(m, 64), triton.cdiv(cout, 64))](dyq, dy_t, m, cout, BLOCK_R=64,
                                                                             BLOCK_C=64)
    partials = torch.empty((split_k, cout, cin * 9), dtype=torch.float32)
    block_n = 128 if cin % 128 == 0 else 64
    grid = (triton.cdiv(cout, 64), triton.cdiv(cin * 9, block_n), split_k)
    fk.conv2d_dw_fp8_kernel.fn[grid](
        xq, dy_t, partials, BATCH=batch, IN_H=h, IN_W=w, CIN=cin, COUT=cout, BLOCK_M=64, BLOCK_N=block_n,
        BLOCK_K=32, SPLIT_K=split_k,
    )
    dw = torch.empty((cout, cin, 3, 3), dtype=torch.bfloat16).contiguous(memory_format=torch.channels_last)
    fk.conv2d_dw_reduce_fp8_kernel[(triton.cdiv(cin * 9 * cout, 256),)](
        partials, dw, sx, sdy, CIN=cin, COUT=cout, SPLIT_K=split_k, BLOCK_SIZE=256
    )
    p = f"{tag}_"
    return {
        p + "dims": np.array([batch, cin, cout, h, w], dtype=np.int64),
        p + "xq": _bytes_u8(_nhwc(xq)),
        p + "wq": _bytes_u8(_nhwc(wq)),
        p + "dyq": _bytes_u8(_nhwc(dyq)),
        p + "scales": np.array([sx.item(), sw.item(), sdy.item()], dtype=np.float32),
        p + "y": _bits_u16(_nhwc(y)),
        p + "dx": _bits_u16(_nhwc(dx)),
        p + "dw": _bits_u16(_nhwc(dw)),
        p + "dyt": _bytes_u8(dy_t),
    }


def main(reference_root: str) -> None:
    sys.path.insert(0, reference_root)
    import diffusion.fp8_kernels as fk  # the reference module

    data: dict[str, np.ndarray] = {}
    data.update(gen_quantize_cases(fk))
    data.update(gen_conv_case(fk, "c128x8", batch=2, cin=128, cout=128, h=8, w=8, seed=1))
    data.update(gen_conv_case(fk, "c256x4", batch=8, cin=256, cout=256, h=4, w=4, seed=2))
    data.update(gen_conv_case(fk, "c128to256x16", batch=1, cin=128, cout=256, h=16, w=16, seed=3))
    # config 2's layer (128 -> 128 at 32x32) at batch 2: the 32x32 halo kernels' shape
    data.update(gen_conv_case(fk, "c128x32", batch=2, cin=128, cout=128, h=32, w=32, seed=4))
    out = HERE / "reference_kernels.npz"
    np.savez_compressed(out, **data)
    print(f"wrote {out} ({out.stat().st_size} bytes, {len(data)} arrays)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {Path(__file__).name} <checkout of the reference repository>")
    main(sys.argv[1])
