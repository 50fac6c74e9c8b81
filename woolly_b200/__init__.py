"""woolly_b200: B200 (sm_100a) quantized transformer forward for woolly.

The compute lives in libwoolly_cuda.so (CUDA kernels + C++ runtime behind the
C ABI in include/woolly_cuda.h); this package is a thin host layer that
mirrors woolly's Rust interfaces.  Nothing here computes on the CPU.
"""
from ._lib import (F16, F32, LAYOUT_A, LAYOUT_B, Q4_0, Q4_1, Q8_0, WoollyError,  # noqa: F401
                   lib)

__version__ = "0.1.0"
