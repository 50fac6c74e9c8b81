"""The C-ABI library loads and exports every symbol include/woolly_cuda.h
declares; host-only entry points behave (CPU only, no compute calls)."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from woolly_b200 import _lib
from woolly_b200.gguf import synth_normal

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    txt = open(os.path.join(ROOT, "include", "woolly_cuda.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(wl_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_header_symbol():
    lib = _lib.lib()
    syms = header_symbols()
    assert len(syms) > 30
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_header():
    assert set(header_symbols()) <= set(_lib.exported_symbols())


def test_version_and_sizes():
    lib = _lib.lib()
    assert b"sm_100a" in lib.wl_version()
    assert [lib.wl_type_size(t) for t in (0, 1, 2, 3, 8)] == [4, 2, 18, 20, 34]
    assert lib.wl_block_size(2) == 32 and lib.wl_block_size(4) == 0


def test_synth_normal_deterministic_and_normal():
    a = synth_normal(1, 2, 200_000, 0.0, 1.0)
    b = synth_normal(1, 2, 200_000, 0.0, 1.0)
    assert np.array_equal(a, b)
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1.0) < 0.01
    assert not np.array_equal(a, synth_normal(1, 3, 200_000))


def test_errors_without_gpu_are_reported():
    # no crash and a status code when asked for a device that is not there
    lib = _lib.lib()
    h = C.c_void_p()
    st = lib.wl_init(999, C.byref(h))
    assert st != 0
    assert lib.wl_last_error()


def test_model_load_rejects_missing_file():
    from woolly_b200.model import model_options
    lib = _lib.lib()
    h = C.c_void_p()
    st = lib.wl_model_load_gguf(None, b"/nonexistent.gguf", C.byref(model_options()), C.byref(h))
    assert st == _lib.WL_ERR_INVALID_ARGUMENT


def test_qtile_bytes_arithmetic():
    """Tiled decode copy size: whole (256-column, 64-row) tiles of
    512 * block_bytes each, equal to the GGUF size for whole tiles."""
    lib = _lib.lib()
    for t, S in ((2, 18), (3, 20), (8, 34)):
        assert lib.wl_qtile_bytes(t, 4096, 4096) == 4096 * 4096 // 32 * S
        assert lib.wl_qtile_bytes(t, 80, 288) == 2 * 2 * 512 * S  # ragged: 2 groups x 2 stages
    assert lib.wl_qtile_bytes(2, 64, 48) == 0   # N % 32 != 0
    assert lib.wl_qtile_bytes(12, 64, 64) == 0  # K-quants need N % 256 == 0
    assert lib.wl_qtile_bytes(12, 80, 512) == 2 * 2 * 512 * 22  # Q4_K: 22 bytes per 32 weights
    assert lib.wl_qtile_bytes(14, 64, 256) == 512 * 40          # Q6_K: 40
    assert lib.wl_qtile_bytes(13, 64, 256) == 0                 # Q5_K: no GEMV
    assert lib.wl_qtile_bytes(2, 0, 64) == 0


def test_new_entry_points_reject_bad_arguments_on_the_host():
    lib = _lib.lib()
    buf = (C.c_uint8 * 64)()
    p = C.cast(buf, C.c_void_p)
    assert lib.wl_qtile_repack(13, p, 64, 256, p, None) == _lib.WL_ERR_UNSUPPORTED
    assert lib.wl_qtile_repack(12, p, 64, 64, p, None) == _lib.WL_ERR_INVALID_ARGUMENT  # N % 256
    assert lib.wl_qtile_repack(2, p, 64, 48, p, None) == _lib.WL_ERR_INVALID_ARGUMENT
    assert lib.wl_qtile_repack(2, None, 64, 64, p, None) == _lib.WL_ERR_INVALID_ARGUMENT
    # K-quant GEMV / GEMM shape rules, checked before any device work
    B = _lib.LAYOUT_B
    assert lib.wl_qgemv(12, B, p, 64, 128, p, 1, p, None) == _lib.WL_ERR_INVALID_ARGUMENT  # N % 256
    assert lib.wl_qgemv(14, B, p, 40, 256, p, 1, p, None) == _lib.WL_ERR_INVALID_ARGUMENT  # K % 16
    assert lib.wl_qgemv(12, _lib.LAYOUT_A, p, 256, 256, p, 1, p, None) == _lib.WL_ERR_UNSUPPORTED
    assert lib.wl_qgemm(14, p, 64, 128, p, 8, p, None) == _lib.WL_ERR_INVALID_ARGUMENT  # N % 256
    assert lib.wl_qgemm_tiled(12, p, 64, 128, p, 0, 8, p, None) == _lib.WL_ERR_INVALID_ARGUMENT
    assert lib.wl_qgemm_tiled(13, p, 64, 256, p, 0, 8, p, None) == _lib.WL_ERR_UNSUPPORTED
    assert lib.wl_qgemv_tiled(2, p, 40, 64, p, 0, 1, p, None) == _lib.WL_ERR_INVALID_ARGUMENT  # K % 16
    assert lib.wl_qgemv_tiled(2, p, 64, 64, p, 0, 0, p, None) == _lib.WL_ERR_INVALID_ARGUMENT  # B = 0
    # tensor-parallel reduce: 1..8 ranks, <= 32 rows, non-null buffers
    args = dict(w=p, dim=64, eps=1e-5, slots=p, counters=p, expect=1, y=p, yp=0, err=None)

    def reduce(h, rows, nranks):
        return lib.wl_tp_reduce_rmsnorm(h, args["w"], rows, args["dim"], args["eps"], args["slots"],
                                        nranks, args["counters"], args["expect"], args["y"],
                                        args["yp"], args["err"], None)
    assert reduce(None, 1, 2) == _lib.WL_ERR_INVALID_ARGUMENT
    assert reduce(p, 1, 9) == _lib.WL_ERR_INVALID_ARGUMENT
    assert reduce(p, 33, 2) == _lib.WL_ERR_INVALID_ARGUMENT
    assert reduce(p, 1, 0) == _lib.WL_ERR_INVALID_ARGUMENT
    assert lib.wl_last_error()
