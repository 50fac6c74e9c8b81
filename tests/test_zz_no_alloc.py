"""wl_qgemv_noalloc: the allocation-free layout-B GEMV (GPU).

Some callers cannot let the library allocate device memory once they are
running, e.g. serving processes that reserve their whole memory budget at
start-up, or hosts whose device allocator belongs to another framework.  This
entry point stages its activations in a fixed array inside the library
instead.  The test calls it through the C ABI twice in a row and checks both
results against wl_qgemv (the allocating entry point) with the GEMV tolerance
used by the op tests; it also checks that sizes above the fixed maximum are
refused.  It lives in its own file so that pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from woolly_b200 import LAYOUT_B, Q4_0, Q4_1, Q8_0, _lib  # noqa: E402
from woolly_b200.gguf import quantize  # noqa: E402

GEMV_TOL = 4e-3  # same bound as tests/test_gpu_ops.py


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _weights(qt, K, N, seed):
    w = (np.random.default_rng(seed).standard_normal(K * N) * 0.02).astype(np.float32)
    return torch.from_numpy(quantize(qt, w)).cuda()


@pytest.mark.parametrize("qt,K,N,B", [(Q4_0, 4096, 4096, 16), (Q4_1, 1024, 768, 5),
                                      (Q8_0, 2048, 512, 33)])
def test_noalloc_matches_allocating_entry(qt, K, N, B):
    lib = _lib.lib()
    W = _weights(qt, K, N, seed=K + N + qt)
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        x = torch.randn(B, K, device="cuda", generator=torch.Generator("cuda").manual_seed(call))
        ref = torch.empty(B, N, device="cuda")
        got = torch.full((B, N), float("nan"), device="cuda")
        _lib.check(lib.wl_qgemv(qt, LAYOUT_B, W.data_ptr(), K, N, x.data_ptr(), B, ref.data_ptr(),
                                stream))
        _lib.check(lib.wl_qgemv_noalloc(qt, W.data_ptr(), K, N, x.data_ptr(), B, got.data_ptr(),
                                        stream))
        torch.cuda.synchronize()
        err = (got - ref).abs().max().item()
        assert err <= GEMV_TOL * ref.abs().max().item() + 1e-6, (call, err)
    # after the first call (set-up done), a call takes no device memory:
    # the device's free memory is unchanged across it
    free0 = torch.cuda.mem_get_info()[0]
    _lib.check(lib.wl_qgemv_noalloc(qt, W.data_ptr(), K, N, x.data_ptr(), B, got.data_ptr(),
                                    stream))
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_rejects_oversize():
    lib = _lib.lib()
    K, N, B = 16384, 256, 33  # B*K > 2^19
    W = torch.zeros(K * N // 32 * 18, dtype=torch.uint8, device="cuda")
    x = torch.zeros(B, K, device="cuda")
    y = torch.zeros(B, N, device="cuda")
    st = lib.wl_qgemv_noalloc(Q4_0, W.data_ptr(), K, N, x.data_ptr(), B, y.data_ptr(), None)
    assert st == _lib.WL_ERR_INVALID_ARGUMENT
    assert b"exceeds" in lib.wl_last_error()
