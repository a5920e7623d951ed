"""GPU test of the allocation-free quantize entry point (collected last on purpose).

``fp8_quantize_current_noalloc`` serves callers that cannot allocate device
memory (runtimes whose device memory is owned by another allocator,
foreign-language hosts reached over FFI without a device allocator): its
scratch is a static array inside libfp8ops.so instead of a caller-provided
workspace.  The test calls it through the C ABI twice in a row, on inputs of
different sizes and ranges, and checks each result against the allocating
entry point ``fp8_quantize_current``: e4m3 bytes and scale must be identical,
the same bar as every quantize test here.  The second, smaller call would pick
up stale maxima if the shared scratch leaked state between calls.
"""

from __future__ import annotations

from ctypes import c_void_p

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ptr(t: torch.Tensor) -> c_void_p:
    return c_void_p(t.data_ptr())


def _allocating(lib, x: torch.Tensor):
    q = torch.empty_like(x, dtype=torch.float8_e4m3fn)
    s = torch.empty((), device=x.device, dtype=torch.float32)
    ws_bytes = lib.fp8_quantize_workspace_bytes(x.numel())
    ws = torch.empty(ws_bytes // 4 + 1, device=x.device, dtype=torch.float32)
    stream = c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    assert lib.fp8_quantize_current(_ptr(x), _ptr(q), _ptr(s), _ptr(ws), ws.numel() * 4, x.numel(), stream) == 0
    return q, s


def _noalloc(lib, x: torch.Tensor):
    q = torch.empty_like(x, dtype=torch.float8_e4m3fn)
    s = torch.empty((), device=x.device, dtype=torch.float32)
    stream = c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    status = lib.fp8_quantize_current_noalloc(_ptr(x), _ptr(q), _ptr(s), x.numel(), stream)
    assert status == 0, status
    return q, s


def test_noalloc_quantize_matches_allocating_entry_point(cuda):
    from fp8_b200 import _lib

    lib = _lib.load()
    g = torch.Generator().manual_seed(123)
    # first call: config-2 sized activation with a large range; second call: a
    # small ragged tensor with a small range (fewer CTAs, smaller amax)
    x1 = (torch.randn(128, 128, 32, 32, generator=g) * 50.0).to(torch.bfloat16).to(cuda)
    x2 = (torch.randn(3, 5, 7, 11, generator=g) * 0.01).to(torch.bfloat16).to(cuda)

    na1 = _noalloc(lib, x1)
    na2 = _noalloc(lib, x2)
    ref1 = _allocating(lib, x1)
    ref2 = _allocating(lib, x2)
    torch.cuda.synchronize()

    for (q, s), (q_ref, s_ref) in ((na1, ref1), (na2, ref2)):
        assert s.item() == s_ref.item()
        assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8))
    assert na2[1].item() < na1[1].item()  # the second scale is its own, not a stale one


def test_noalloc_quantize_unaligned_views_take_the_scalar_path(cuda):
    """Views that start one element past a 16-byte boundary go through the scalar
    amax / cast kernels; two such calls in a row through the shared scratch must
    still equal the allocating entry point bit for bit."""
    from fp8_b200 import _lib

    lib = _lib.load()
    g = torch.Generator().manual_seed(321)
    base1 = (torch.randn(64 * 128 * 16 * 16 + 1, generator=g) * 3.0).to(torch.bfloat16).to(cuda)
    base2 = (torch.randn(4099, generator=g) * 1e-3).to(torch.bfloat16).to(cuda)
    x1, x2 = base1[1:], base2[1:]
    assert x1.data_ptr() % 16 != 0 and x2.data_ptr() % 16 != 0

    na1 = _noalloc(lib, x1)
    na2 = _noalloc(lib, x2)
    ref1 = _allocating(lib, x1)
    ref2 = _allocating(lib, x2)
    torch.cuda.synchronize()

    for (q, s), (q_ref, s_ref) in ((na1, ref1), (na2, ref2)):
        assert s.item() == s_ref.item()
        assert torch.equal(q.view(torch.uint8), q_ref.view(torch.uint8))
    assert na2[1].item() < na1[1].item()
