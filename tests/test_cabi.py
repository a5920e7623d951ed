"""CPU tests of the C ABI: the library loads, exports every declared symbol, and
validates arguments on the host (no CUDA call is reached for invalid sizes)."""

from __future__ import annotations

import ctypes
import re
from ctypes import c_void_p
from pathlib import Path

import pytest

from fp8_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "fp8ops.h"


def _declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|size_t)\s+(fp8_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_functions():
    names = _declared_functions()
    assert "fp8_conv3x3_fwd" in names and "fp8_quantize_current" in names and len(names) >= 15


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in _declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert sorted(_lib.exported_symbols()) == _declared_functions()


def test_abi_version():
    assert _lib.load().fp8_abi_version() == 4


def _status_and_message(fn, *args):
    status = fn(*args)
    code, msg = _lib.last_error()
    return status, code, msg


def test_conv_rejects_unsupported_channels_without_touching_cuda():
    lib = _lib.load()
    null = c_void_p(0)
    status, code, msg = _status_and_message(
        lib.fp8_conv3x3_fwd, null, null, null, null, null, null, 0, 2, 8, 8, 100, 128, null
    )
    assert status == _lib.FP8_ERR_UNSUPPORTED and code == status and "multiples of 128" in msg


def test_conv_rejects_untileable_spatial():
    lib = _lib.load()
    null = c_void_p(0)
    status, _, msg = _status_and_message(lib.fp8_conv3x3_dgrad, null, null, null, null, null, 2, 7, 7, 128, 128,
                                         null)
    assert status == _lib.FP8_ERR_UNSUPPORTED and "tileable" in msg


def test_conv_rejects_nonpositive_sizes():
    lib = _lib.load()
    null = c_void_p(0)
    status, _, _ = _status_and_message(lib.fp8_conv3x3_wgrad, null, null, null, null, null, 0, 8, 8, 128, 128, 0,
                                       null, 0, null)
    assert status == _lib.FP8_ERR_INVALID_ARGUMENT


def test_gemm_rejects_bad_k_and_n():
    lib = _lib.load()
    null = c_void_p(0)
    assert lib.fp8_gemm(null, null, null, null, null, null, 0, 16, 64, 10, null) == _lib.FP8_ERR_UNSUPPORTED
    assert lib.fp8_gemm(null, null, null, null, null, null, 0, 16, 40, 64, null) == _lib.FP8_ERR_UNSUPPORTED
    assert lib.fp8_gemm_wgrad(null, null, null, null, null, 16, 64, 128, 0, null, 0, null) == \
        _lib.FP8_ERR_UNSUPPORTED


def test_quantize_rejects_negative_n_and_null_scale():
    lib = _lib.load()
    null = c_void_p(0)
    assert lib.fp8_quantize_current(null, null, null, null, 0, -1, null) == _lib.FP8_ERR_INVALID_ARGUMENT
    status, _, msg = _status_and_message(lib.fp8_quantize_delayed, null, null, null, null, null, 0, 4, null)
    assert status == _lib.FP8_ERR_INVALID_ARGUMENT and "prev_scale" in msg


def test_tile_override_validation():
    lib = _lib.load()
    assert lib.fp8_set_tile_override(3, 0, 0) == _lib.FP8_ERR_INVALID_ARGUMENT
    assert lib.fp8_set_tile_override(0, 96, 0) == _lib.FP8_ERR_INVALID_ARGUMENT
    assert lib.fp8_set_tile_override(0, 0, 0) == _lib.FP8_OK
    assert _lib.last_error() == (0, "")


def test_check_raises_with_library_message():
    lib = _lib.load()
    with pytest.raises(RuntimeError, match="bm_sub"):
        _lib.check(lib.fp8_set_tile_override(5, 0, 0), "fp8_set_tile_override")


def test_workspace_queries_are_host_only():
    lib = _lib.load()
    # unsupported geometry -> 0 bytes, no CUDA needed
    assert lib.fp8_conv3x3_wgrad_workspace_bytes(2, 7, 7, 128, 128, 0) == 0
    assert lib.fp8_gemm_wgrad_workspace_bytes(16, 100, 128, 0) == 0
    # one fp32 accumulator of Cout * 9 * Cin, whatever the split count
    assert lib.fp8_conv3x3_wgrad_workspace_bytes(2, 8, 8, 128, 128, 1) == 128 * 9 * 128 * 4
    assert lib.fp8_conv3x3_wgrad_workspace_bytes(2, 8, 8, 128, 256, 7) == 256 * 9 * 128 * 4
    assert lib.fp8_gemm_wgrad_workspace_bytes(300, 256, 128, 0) == 256 * 128 * 4


def test_python_ops_have_no_cpu_path():
    import torch

    from fp8_b200 import fp8_kernels, ops

    x = torch.zeros(1, 128, 8, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.quantize_current(x)
    with pytest.raises(AssertionError):  # the reference API asserts is_cuda (fp8_kernels.py:560-562)
        fp8_kernels.quantize_fp8(x)


def test_reference_api_names_present():
    from fp8_b200 import fp8_kernels

    for name in [
        "FP8_DTYPE", "FP8_MAX_E4M3", "SUPPORTED_UNET_SHAPES", "quantize_fp8", "quantize_fp8_delayed",
        "conv2d_fwd_fp8", "conv2d_fwd_fp8_prequantized", "conv2d_fwd_fp8_delayed", "conv2d_bwd_input_fp8",
        "conv2d_bwd_input_fp8_prequantized", "conv2d_bwd_weight_fp8", "conv2d_bwd_weight_fp8_prequantized",
        "Conv2dFP8Specialized", "triton_conv2d_fp8", "torch_checks_conv", "fwd_shapes", "xgrad_shapes",
        "wgrad_shapes", "torch_checks_scale",
    ]:
        assert hasattr(fp8_kernels, name), name
    assert fp8_kernels.FP8_MAX_E4M3 == 448.0
    assert len(fp8_kernels.SUPPORTED_UNET_SHAPES) == 9


def test_ctypes_signatures_match_header_arity():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, (_, args) in _lib._SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\((.*?)\)\s*;", text, flags=re.S)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), (name, len(params), len(args))
    assert ctypes.sizeof(ctypes.c_size_t) == 8


def test_dgrad_w_workspace_sizing_and_check():
    """The data-grad on the forward's weights needs no workspace where it reads
    them in place (Cout = 128 at 32x32 / 16x16) and 9*Cin*Cout bytes otherwise;
    a missing workspace is rejected on the host."""
    lib = _lib.load()
    assert lib.fp8_conv3x3_dgrad_w_workspace_bytes(4, 32, 32, 256, 128) == 0
    assert lib.fp8_conv3x3_dgrad_w_workspace_bytes(4, 16, 16, 128, 128) == 0
    assert lib.fp8_conv3x3_dgrad_w_workspace_bytes(4, 32, 32, 128, 256) == 9 * 128 * 256
    assert lib.fp8_conv3x3_dgrad_w_workspace_bytes(4, 8, 8, 256, 256) == 9 * 256 * 256
    fake = c_void_p(1 << 20)  # 16-byte aligned, never dereferenced: the call fails before any device work
    status, code, msg = _status_and_message(
        lib.fp8_conv3x3_dgrad_w, fake, fake, fake, fake, fake, 2, 8, 8, 256, 256, c_void_p(0), 0, c_void_p(0)
    )
    assert status == _lib.FP8_ERR_WORKSPACE and code == status and "workspace" in msg


def test_layer_norm_rejects_bad_channels_without_touching_cuda():
    lib = _lib.load()
    fake = c_void_p(1 << 20)
    status, code, msg = _status_and_message(
        lib.fp8_layer_norm_fwd, fake, 0, fake, fake, ctypes.c_float(1e-5), fake, fake, 64, 12, c_void_p(0)
    )
    assert status == _lib.FP8_ERR_UNSUPPORTED and code == status and "c % 8" in msg
    assert lib.fp8_layer_norm_workspace_bytes(0, 256) == 0


def test_resample_rejects_bad_channels_without_touching_cuda():
    lib = _lib.load()
    fake = c_void_p(1 << 20)
    status, code, msg = _status_and_message(lib.fp8_up_cat, fake, 0, fake, 0, fake, 1, 2, 8, 8, 12, 8, 2, c_void_p(0))
    assert status == _lib.FP8_ERR_UNSUPPORTED and code == status and "multiples of 8" in msg
    status, code, msg = _status_and_message(lib.fp8_resample_down2, fake, 0, fake, 2, 7, 8, 16, c_void_p(0))
    assert status == _lib.FP8_ERR_UNSUPPORTED and "even" in msg


def test_cast_batch_validates_without_touching_cuda():
    lib = _lib.load()
    arr = (c_void_p * 1)(c_void_p(1 << 20))
    n = (ctypes.c_int64 * 1)(16)
    status, code, msg = _status_and_message(lib.fp8_cast_batch, 65, arr, arr, n, 1, c_void_p(0))
    assert status == _lib.FP8_ERR_UNSUPPORTED and code == status and "1..64" in msg
    odd = (c_void_p * 1)(c_void_p((1 << 20) + 2))  # fp32 source 2 bytes off alignment
    status, code, msg = _status_and_message(lib.fp8_cast_batch, 1, odd, arr, n, 1, c_void_p(0))
    assert status == _lib.FP8_ERR_INVALID_ARGUMENT and "misaligned" in msg


def test_new_fused_entry_points_validate_without_touching_cuda():
    """The producer-side dY casts, the paired up_cat and the widened dW reject bad arguments before any
    CUDA call (status and message, no device work)."""
    lib = _lib.load()
    fake = c_void_p(1 << 20)
    odd = c_void_p((1 << 20) + 8)
    null = c_void_p(0)
    # join backward + quantize: n not a multiple of 8; a NULL / misaligned e4m3 output; a bad history
    status, code, msg = _status_and_message(lib.fp8_add_scale_bwd_quant, fake, 0, fake, 0, fake, fake, fake, 16,
                                            fake, fake, 12, ctypes.c_float(0.7), fake, 64, null)
    assert status == _lib.FP8_ERR_UNSUPPORTED and code == status and "multiple of 8" in msg
    status, code, msg = _status_and_message(lib.fp8_add_scale_bwd_quant, fake, 0, fake, 0, fake, odd, fake, 16,
                                            fake, fake, 64, ctypes.c_float(0.7), fake, 64, null)
    assert status == _lib.FP8_ERR_INVALID_ARGUMENT and "dbq" in msg
    status, code, msg = _status_and_message(lib.fp8_add_scale_bwd_quant, fake, 0, fake, 0, fake, fake, fake, 0,
                                            fake, fake, 64, ctypes.c_float(0.7), fake, 64, null)
    assert status == _lib.FP8_ERR_INVALID_ARGUMENT and "history" in msg
    assert lib.fp8_add_scale_bwd_quant_workspace_bytes(12) == 0
    # group-norm backward + quantize: unsupported channel count
    status, code, msg = _status_and_message(
        lib.fp8_gn_act_bwd_quant, fake, fake, fake, fake, null, 0, null, ctypes.c_float(0.0), ctypes.c_float(1e-5),
        fake, fake, fake, fake, fake, 16, fake, fake, 2, 64, 12, 4, fake, 1 << 20, null)
    assert status == _lib.FP8_ERR_UNSUPPORTED and "c % 8" in msg
    # paired up_cat: a misaligned bf16 copy
    status, code, msg = _status_and_message(lib.fp8_up_cat_pair, fake, 0, fake, 0, fake, odd, 1, 8, 8, 16, 16, 2, null)
    assert status == _lib.FP8_ERR_INVALID_ARGUMENT and "y_bf16" in msg
    status, code, msg = _status_and_message(lib.fp8_up_cat_pair_bwd, fake, null, fake, 0, fake, 0, 1, 8, 8, 16, 16, 2,
                                            null)
    assert status == _lib.FP8_ERR_INVALID_ARGUMENT and "dy_bf16" in msg
    # widened dW: unsupported channels, as fp8_conv3x3_wgrad
    status, code, msg = _status_and_message(lib.fp8_conv3x3_wgrad_f32, null, null, null, null, null, 2, 8, 8, 100, 128,
                                            0, null, 0, null)
    assert status == _lib.FP8_ERR_UNSUPPORTED and "multiples of 128" in msg


def test_weight_transpose_batch_validates_without_touching_cuda():
    lib = _lib.load()
    arr = (c_void_p * 1)(c_void_p(1 << 20))
    dims = (ctypes.c_int * 1)(128)
    bad = (ctypes.c_int * 1)(96)
    status, code, msg = _status_and_message(lib.fp8_conv_weight_transpose_batch, 65, arr, arr, dims, dims, c_void_p(0))
    assert status == _lib.FP8_ERR_UNSUPPORTED and "1..64" in msg
    status, code, msg = _status_and_message(lib.fp8_conv_weight_transpose_batch, 1, arr, arr, bad, dims, c_void_p(0))
    assert status == _lib.FP8_ERR_UNSUPPORTED and "multiples of 64" in msg


def test_selftest_wait_validates_without_touching_cuda():
    lib = _lib.load()
    null = c_void_p(0)
    for limit in (0, 2_000_000_000):
        status, code, msg = _status_and_message(lib.fp8_selftest_wait_timeout, ctypes.c_uint64(limit), c_void_p(16),
                                                null)
        assert status == _lib.FP8_ERR_INVALID_ARGUMENT and "limit_ns" in msg
    status, code, msg = _status_and_message(lib.fp8_selftest_wait_timeout, ctypes.c_uint64(1000), null, null)
    assert status == _lib.FP8_ERR_INVALID_ARGUMENT and "returned" in msg


def test_attention_validates_without_touching_cuda():
    lib = _lib.load()
    null = c_void_p(0)
    # head_dim 32, sequence 300, sequence 40: rejected before any CUDA call
    for head_dim, seq in ((32, 256), (64, 300), (64, 40)):
        status, code, msg = _status_and_message(lib.fp8_attention_fwd, c_void_p(16), c_void_p(16), c_void_p(16),
                                                c_void_p(16), 2, seq, 4, head_dim, 768, 256, null)
        assert status == _lib.FP8_ERR_UNSUPPORTED, (head_dim, seq, msg)
    status, code, msg = _status_and_message(lib.fp8_attention_bwd, c_void_p(16), c_void_p(16), c_void_p(16),
                                            c_void_p(16), c_void_p(16), c_void_p(16), 2, 256, 4, 64, 700, 256, null)
    assert status == _lib.FP8_ERR_INVALID_ARGUMENT and "strides" in msg
