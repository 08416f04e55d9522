"""B200 (sm_100a) quantized decode GEMV -- host-side Python mirror of the C-ABI.

The kernels and the C-ABI live in libqgemv_b200.so (csrc/, include/qgemv_b200.h).
`ops` wraps the entry points for torch CUDA tensors; `packs` holds the resident-pack
byte layouts and the seeded synthetic pack generator.
"""

from . import packs  # noqa: F401
from ._lib import CudaError, call, check, header_functions, lib  # noqa: F401

__all__ = ["packs", "lib", "call", "check", "header_functions", "CudaError"]
