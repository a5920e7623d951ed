"""Failure path of the bounded device waits, exercised without faulting the GPU.

Every mbarrier wait in this library's kernels gives up after a wall-time limit,
records an error code in the device error word, raises the CTA's abort flag and
returns.  Here a self-test kernel waits on a barrier that nothing arrives on,
through that same wait with a 50 ms limit: the wait must run out, the code must
read back through ``fp8_device_error`` (which also clears it), and the context
must stay usable for the next op."""

from __future__ import annotations

import ctypes
import time

import pytest
import torch

import fp8_oracle as oracle

pytestmark = pytest.mark.gpu

SELFTEST_CODE = 199


def test_bounded_wait_runs_out_and_reports(cuda):
    from fp8_b200 import _lib, ops

    assert _lib.device_error() == 0
    returned = torch.zeros(1, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    t0 = time.perf_counter()
    _lib.call("fp8_selftest_wait_timeout", ctypes.c_uint64(50_000_000), ctypes.c_void_p(returned.data_ptr()),
              ctypes.c_void_p(stream))
    code = _lib.device_error(stream)  # synchronises the stream
    elapsed = time.perf_counter() - t0
    assert code == SELFTEST_CODE
    assert int(returned.item()) == 1  # the waiting thread came back with "gave up"
    assert 0.04 <= elapsed < 10.0, elapsed
    assert _lib.device_error(stream) == 0  # read-and-clear

    # the context is still usable: a quantize right after gives the oracle's bytes
    x = torch.randn(4, 128, 8, 8, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16)
    q, s = ops.quantize_current(x.to(cuda))
    qr, sr = oracle.quantize_tensor(x)
    assert torch.equal(q.cpu().view(torch.uint8), qr.view(torch.uint8))
    assert float(s.item()) == float(sr.item())
    assert _lib.device_error(stream) == 0
