"""woolly_b200: B200 (sm_100a) quantized transformer forward for woolly.

The compute lives in libwoolly_cuda.so (CUDA kernels + C++ runtime behind the
C ABI in include/woolly_cuda.h); this package is a thin host layer that
mirrors woolly's Rust interfaces.  All model compute runs on the GPU; the
only host arithmetic is engine.py's restatement of the server's sampling
rules, for callers that keep logits on the host.
"""
from ._lib import (F16, F32, LAYOUT_A, LAYOUT_B, Q4_0, Q4_1, Q4_K, Q6_K, Q8_0,  # noqa: F401
                   WoollyError, lib)

__version__ = "0.1.0"
