"""fp8_b200 — B200 (sm_100a) FP8 hot path of the diffusion-profiled DDPM UNet.

* :mod:`fp8_b200.fp8_kernels` — drop-in for the reference module
  ``diffusion/fp8_kernels.py`` (same names and semantics).
* :mod:`fp8_b200.ops` — the torch custom ops over the C ABI (include/fp8ops.h).
* :mod:`fp8_b200.linear` — the scaled FP8 linear (no reference kernel).

Importing the package loads ``libfp8ops.so``; a missing library is an error,
there is no CPU or Triton fallback.
"""

from . import _lib

_lib.load()

from . import ops  # noqa: E402
from . import fp8_kernels  # noqa: E402

__all__ = ["ops", "fp8_kernels"]
