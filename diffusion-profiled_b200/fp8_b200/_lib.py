"""ctypes binding of ``libfp8ops.so`` (the C ABI declared in include/fp8ops.h).

This is the only place Python touches the native library.  Every wrapper raises
``RuntimeError`` carrying the library's own error message when a call returns a
non-zero status.  There is no fallback: if the library is missing the import
of :mod:`fp8_b200` fails loudly.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import c_int, c_int64, c_size_t, c_void_p, POINTER, c_float, c_char_p

from .build import LIB_PATH

FP8_OK = 0
FP8_ERR_INVALID_ARGUMENT = 1
FP8_ERR_UNSUPPORTED = 2
FP8_ERR_CUDA = 3
FP8_ERR_WORKSPACE = 4

EPILOGUE_NONE = 0
EPILOGUE_BIAS = 1
EPILOGUE_BIAS_SILU = 2

# name -> (restype, argtypes); mirrors include/fp8ops.h one to one.
_SIGNATURES: dict[str, tuple] = {
    "fp8_abi_version": (c_int, []),
    "fp8_last_error": (c_int, [c_char_p, c_size_t]),
    "fp8_device_error": (c_int, [POINTER(c_int), c_void_p]),
    "fp8_sm_count": (c_int, [POINTER(c_int)]),
    "fp8_selftest_wait_timeout": (c_int, [ctypes.c_uint64, c_void_p, c_void_p]),
    "fp8_attention_fwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
                                  c_void_p]),
    "fp8_attention_bwd": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                                  c_int, c_int, c_int, c_void_p]),
    "fp8_kernel_launch_count": (c_int, [POINTER(ctypes.c_ulonglong)]),
    "fp8_quantize_workspace_bytes": (c_size_t, [c_int64]),
    "fp8_quantize_current": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_int64, c_void_p]),
    "fp8_quantize_current_noalloc": (c_int, [c_void_p, c_void_p, c_void_p, c_int64, c_void_p]),
    "fp8_quantize_delayed": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_size_t, c_int64, c_void_p],
    ),
    "fp8_transpose_2d": (c_int, [c_void_p, c_void_p, c_int64, c_int64, c_void_p]),
    "fp8_conv_weight_transpose": (c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p]),
    "fp8_conv3x3_fwd": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int,
         c_void_p],
    ),
    "fp8_conv3x3_dgrad": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p],
    ),
    "fp8_conv3x3_dgrad_w_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    "fp8_conv3x3_dgrad_w": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
         c_void_p],
    ),
    "fp8_conv3x3_wgrad_workspace_bytes": (c_size_t, [c_int, c_int, c_int, c_int, c_int, c_int]),
    "fp8_conv3x3_wgrad": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
         c_size_t, c_void_p],
    ),
    "fp8_conv3x3_wgrad_f32": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
         c_size_t, c_void_p],
    ),
    "fp8_gemm": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64, c_void_p],
    ),
    "fp8_gemm_wgrad_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int]),
    "fp8_gemm_wgrad": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int, c_void_p, c_size_t,
         c_void_p],
    ),
    "fp8_set_tile_override": (c_int, [c_int, c_int, c_int]),
    "fp8_set_quantize_override": (c_int, [c_int, c_int]),
    "fp8_quantize_multi_workspace_bytes": (c_size_t, [c_int]),
    "fp8_quantize_current_multi": (c_int, [c_int, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p),
                                           POINTER(c_int64), c_void_p, c_size_t, c_void_p]),
    "fp8_gn_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "fp8_gn_act_fwd": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_float, c_float,
                               c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p]),
    "fp8_layer_norm_fwd": (
        c_int, [c_void_p, c_int, c_void_p, c_void_p, c_float, c_void_p, c_void_p, c_int64, c_int, c_void_p]),
    "fp8_layer_norm_workspace_bytes": (c_size_t, [c_int64, c_int]),
    "fp8_layer_norm_bwd": (
        c_int,
        [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int, c_void_p,
         c_size_t, c_void_p],
    ),
    "fp8_gn_param_grads": (
        c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "fp8_resample_down2": (c_int, [c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_void_p]),
    "fp8_resample_down2_bwd": (c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p]),
    "fp8_up_cat": (
        c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                c_void_p]),
    "fp8_up_cat_bwd": (
        c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int,
                c_void_p]),
    "fp8_add_scale_bwd_quant_workspace_bytes": (c_size_t, [c_int64]),
    "fp8_add_scale_bwd_quant": (
        c_int,
        [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int64,
         c_float, c_void_p, c_size_t, c_void_p],
    ),
    "fp8_gn_act_bwd_quant_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "fp8_gn_act_bwd_quant": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_float, c_float, c_void_p, c_void_p,
         c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
         c_void_p],
    ),
    "fp8_gn_act_bwd_accumulate": (
        c_int,
        [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_float, c_float, c_void_p,
         c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "fp8_conv_weight_transpose_batch": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "fp8_cast_batch": (c_int, [c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p]),
    "fp8_up_cat_pair": (
        c_int,
        [c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p],
    ),
    "fp8_up_cat_pair_bwd": (
        c_int,
        [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p],
    ),
    "fp8_quantize_delayed_window": (
        c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_size_t, c_int64,
                c_void_p]),
    "fp8_gn_act_quant_fwd_window": (
        c_int,
        [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_float, c_float, c_void_p, c_int, c_void_p,
         c_int, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "fp8_quantize_weights_delayed_workspace_bytes": (c_size_t, [c_int, POINTER(c_int64)]),
    "fp8_quantize_weights_delayed": (
        c_int,
        [c_int, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_int64), POINTER(c_void_p), c_int, POINTER(c_void_p),
         POINTER(c_void_p), c_void_p, c_size_t, c_void_p],
    ),
    "fp8_adamw_ema_workspace_bytes": (c_size_t, [c_int, POINTER(c_int64)]),
    "fp8_adamw_ema_step": (
        c_int,
        [c_int, POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p), POINTER(c_void_p),
         POINTER(c_int64), c_void_p, c_float, c_float, c_float, c_float, c_float, c_float, c_float, c_void_p,
         c_size_t, c_void_p],
    ),
    "fp8_add_scale": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int64, c_float, c_void_p]),
    "fp8_add_scale_bwd": (c_int, [c_void_p, c_int, c_void_p, c_int, c_void_p, c_int, c_int64, c_float, c_void_p]),
    "fp8_gn_act_quant_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "fp8_gn_act_quant_fwd": (
        c_int,
        [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_float, c_float, c_void_p, c_void_p,
         c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p],
    ),
    "fp8_gn_act_bwd": (c_int, [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_float,
                               c_float, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                               c_size_t, c_void_p]),
    "fp8_set_conv_algo": (c_int, [c_int]),
    "fp8_set_pdl": (c_int, [c_int]),
    "fp8_set_empty_tensor_history": (c_int, [c_int]),
    "fp8_set_quantize_resident": (c_int, [c_int]),
    "fp8_set_wgrad_fused": (c_int, [c_int]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the in-tree library (once) and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with fp8_b200.build.build_library() "
                    "(or __graft_entry__.build()); there is no fallback implementation"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> tuple[int, str]:
    buf = ctypes.create_string_buffer(512)
    code = load().fp8_last_error(buf, len(buf))
    return code, buf.value.decode(errors="replace")


def check(status: int, what: str) -> None:
    if status != FP8_OK:
        code, msg = last_error()
        raise RuntimeError(f"{what} failed (status {status}): {msg}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def device_error(stream: int = 0) -> int:
    code = c_int(0)
    check(load().fp8_device_error(ctypes.byref(code), c_void_p(stream)), "fp8_device_error")
    return code.value


def sm_count() -> int:
    out = c_int(0)
    check(load().fp8_sm_count(ctypes.byref(out)), "fp8_sm_count")
    return out.value


def kernel_launch_count() -> int:
    out = ctypes.c_ulonglong(0)
    check(load().fp8_kernel_launch_count(ctypes.byref(out)), "fp8_kernel_launch_count")
    return out.value


def set_tile_override(bm_sub: int = 0, bn: int = 0, wgrad_group: int = 0) -> None:
    check(load().fp8_set_tile_override(bm_sub, bn, wgrad_group), "fp8_set_tile_override")


def set_pdl(mode: int = 0) -> None:
    """0: plain stream order (the default); 1: programmatic dependent launch of
    the tensor-core kernels; 2: of every kernel."""
    check(load().fp8_set_pdl(int(mode)), "fp8_set_pdl")


def set_empty_tensor_history(mode: int = 0) -> None:
    """0: an all-zero tensor records its scale 1.0 in the delayed-scaling histories (the
    reference); 1: it records 0.0 (adds nothing to the history max)."""
    check(load().fp8_set_empty_tensor_history(int(mode)), "fp8_set_empty_tensor_history")


def set_quantize_resident(enable: bool = True) -> None:
    """Current-scaling quantize as one shared-memory-resident launch where it applies (default)
    or always as two passes."""
    check(load().fp8_set_quantize_resident(int(enable)), "fp8_set_quantize_resident")


def set_wgrad_fused(enable: bool = False) -> None:
    """Weight gradients with the accumulator conversion folded into the split-K launch, or as a
    second launch (the default)."""
    check(load().fp8_set_wgrad_fused(int(enable)), "fp8_set_wgrad_fused")


def set_conv_algo(algo: int = 0) -> None:
    check(load().fp8_set_conv_algo(algo), "fp8_set_conv_algo")


def set_quantize_override(amax_blocks_per_sm: int = 0, cast_blocks_per_sm: int = 0) -> None:
    check(load().fp8_set_quantize_override(amax_blocks_per_sm, cast_blocks_per_sm), "fp8_set_quantize_override")


__all__ = [
    "load",
    "call",
    "check",
    "last_error",
    "device_error",
    "sm_count",
    "set_tile_override",
    "exported_symbols",
    "c_float",
]
