"""ctypes wrapper of the CPU oracle (oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs as the checker / timed CPU restatement of
woolly's path.  The product (woolly_b200/) never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")

F32, F16, Q4_0, Q4_1, Q8_0 = 0, 1, 2, 3, 8
Q4_K, Q6_K = 12, 14


def build() -> str:
    src = [os.path.join(HERE, f) for f in ("oracle.c", "synth.c", "oracle.h", "Makefile")]
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(map(os.path.getmtime, src)):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


class Opts(C.Structure):
    _fields_ = [("rope", C.c_int), ("window", C.c_int), ("swiglu", C.c_int),
                ("threads", C.c_int), ("max_layers", C.c_int), ("layout_a", C.c_int)]


class SynthCfg(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("layers", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("ff", C.c_uint32), ("vocab", C.c_uint32),
                ("context_length", C.c_uint32), ("weight_type", C.c_uint32),
                ("output_type", C.c_uint32), ("sliding_window", C.c_uint32),
                ("rope_theta", C.c_float), ("norm_eps", C.c_float), ("seed", C.c_uint64),
                ("vd_type", C.c_uint32), ("embd_type", C.c_uint32)]


_lib = None
P = C.c_void_p
_SIGS = {
    "or_half_to_float": (C.c_float, [C.c_uint16]),
    "or_block_size": (C.c_size_t, [C.c_int]),
    "or_type_size": (C.c_size_t, [C.c_int]),
    "or_align_offset": (C.c_uint64, [C.c_uint64, C.c_uint64]),
    "or_dequantize": (C.c_int, [P, C.c_size_t, C.c_int, C.c_size_t, P]),
    "or_quantized_matvec": (C.c_int, [C.c_int, P, P, P, C.c_size_t, C.c_size_t]),
    "or_gguf_open_mem": (C.c_int, [P, C.c_size_t, C.POINTER(P)]),
    "or_gguf_close": (None, [P]),
    "or_model_load": (C.c_int, [C.c_char_p, C.POINTER(Opts), C.POINTER(P)]),
    "or_model_free": (None, [P]),
    "or_model_dims": (None, [P] + [C.POINTER(C.c_int)] * 6),
    "or_kv_new": (P, [P, C.c_int]),
    "or_kv_free": (None, [P]),
    "or_kv_len": (C.c_int, [P]),
    "or_kv_fill_synthetic": (C.c_int, [P, C.c_int, C.c_uint64]),
    "or_forward": (C.c_int, [P, P, P, C.c_int, P, C.c_int]),
    "or_decode_batch": (C.c_int, [P, C.POINTER(P), C.c_int, P, P]),
    "or_synth_gguf": (C.c_int, [C.c_char_p, C.POINTER(SynthCfg)]),
    "or_rms_norm": (None, [P, P, C.c_int, C.c_int, C.c_float, P]),
    "or_swiglu": (None, [P, P, C.c_size_t, C.c_int, P]),
    "or_rope_neox": (None, [P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]),
    "or_matmul_b": (None, [P, C.c_int, C.c_int, P, C.c_int, P]),
    "or_attention": (None, [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P]),
}


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        build()
        h = C.CDLL(LIB)
        for n, (r, a) in _SIGS.items():
            f = getattr(h, n)
            f.restype, f.argtypes = r, a
        _lib = h
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def half_to_float(h: int) -> float:
    return lib().or_half_to_float(h)


def synth_gguf(path: str, *, hidden: int, layers: int, heads: int, kv_heads: int, ff: int,
               vocab: int, weight_type: int = Q4_0, output_type: int | None = None,
               tied: bool = False, context_length: int = 4096, sliding_window: int = 0,
               rope_theta: float = 10000.0, norm_eps: float = 1e-5, seed: int = 0,
               vd_type: int = 0, embd_type: int = 0) -> str:
    """The seeded LLaMA-shape GGUF of the product's writer, written by the
    oracle's own C writer (synth.c), so CPU-only legs never load the product
    library."""
    cfg = SynthCfg(hidden, layers, heads, kv_heads, ff, vocab, context_length, weight_type,
                   0xFFFFFFFF if tied else (weight_type if output_type is None else output_type),
                   sliding_window, rope_theta, norm_eps, seed, vd_type, embd_type)
    st = lib().or_synth_gguf(str(path).encode(), C.byref(cfg))
    if st:
        raise ValueError(f"or_synth_gguf status {st}")
    return str(path)


def dequantize(data: bytes | np.ndarray, ggml_type: int, n: int) -> np.ndarray:
    buf = np.frombuffer(bytes(data), dtype=np.uint8) if not isinstance(data, np.ndarray) else \
        np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    st = lib().or_dequantize(buf.ctypes.data if buf.size else None, buf.size, ggml_type, n,
                             out.ctypes.data)
    if st:
        raise ValueError(f"or_dequantize status {st}")
    return out


def quantized_matvec(ggml_type: int, blocks: np.ndarray, x: np.ndarray, m: int, k: int) -> np.ndarray:
    b = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = _f32(x)
    y = np.empty(m, dtype=np.float32)
    st = lib().or_quantized_matvec(ggml_type, b.ctypes.data, x.ctypes.data, y.ctypes.data, m, k)
    if st:
        raise ValueError(f"or_quantized_matvec status {st}")
    return y


def gguf_status(data: bytes) -> int:
    """Parse status of a GGUF image (0 = ok)."""
    buf = C.create_string_buffer(data, len(data)) if data else None
    h = P()
    st = lib().or_gguf_open_mem(buf, len(data), C.byref(h))
    if st == 0:
        lib().or_gguf_close(h)
    return st


def rms_norm(x, w, eps) -> np.ndarray:
    x = _f32(x)
    w = _f32(w)
    d = w.size
    y = np.empty_like(x)
    lib().or_rms_norm(x.ctypes.data, w.ctypes.data, x.size // d, d, eps, y.ctypes.data)
    return y


def swiglu(g, u, mode: int = 0) -> np.ndarray:
    g, u = _f32(g), _f32(u)
    out = np.empty_like(g)
    lib().or_swiglu(g.ctypes.data, u.ctypes.data, g.size, mode, out.ctypes.data)
    return out


def rope_neox(x, positions, batch, seq, heads, hd, base) -> np.ndarray:
    y = _f32(x).copy()
    pos = np.ascontiguousarray(positions, dtype=np.uint64)
    lib().or_rope_neox(y.ctypes.data, pos.ctypes.data, batch, seq, heads, hd, base)
    return y


def matmul_b(x, W, K, N) -> np.ndarray:
    x, W = _f32(x), _f32(W)
    rows = x.size // K
    y = np.empty((rows, N), dtype=np.float32)
    lib().or_matmul_b(x.ctypes.data, rows, K, W.ctypes.data, N, y.ctypes.data)
    return y


def attention(q, k, v, rows, past, heads, kv_heads, hd, window=0) -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty((rows, heads * hd), dtype=np.float32)
    lib().or_attention(q.ctypes.data, k.ctypes.data, v.ctypes.data, rows, past, heads, kv_heads,
                       hd, window, out.ctypes.data)
    return out


class Model:
    """Oracle model: every weight dequantized to f32, KV-cache forward."""

    def __init__(self, path: str, rope: int = 0, window: int = 0, swiglu: int = 0,
                 threads: int = 0, max_layers: int = 0, layout_a: int = 0):
        self._o = Opts(rope, window, swiglu, threads, max_layers, layout_a)
        self._h = P()
        st = lib().or_model_load(str(path).encode(), C.byref(self._o), C.byref(self._h))
        if st:
            raise ValueError(f"or_model_load status {st}")
        dims = [C.c_int() for _ in range(6)]
        lib().or_model_dims(self._h, *[C.byref(d) for d in dims])
        (self.hidden, self.layers, self.heads, self.kv_heads, self.ff, self.vocab) = \
            [d.value for d in dims]

    def close(self):
        if self._h:
            lib().or_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def new_kv(self, max_ctx: int) -> "KV":
        return KV(self, max_ctx)

    def forward(self, kv: "KV", ids, all_rows: bool = True) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        rows = ids.size if all_rows else 1
        out = np.empty((rows, self.vocab), dtype=np.float32)
        st = lib().or_forward(self._h, kv._h, ids.ctypes.data, ids.size, out.ctypes.data,
                              1 if all_rows else 0)
        if st:
            raise ValueError(f"or_forward status {st}")
        return out

    def decode_batch(self, kvs, ids) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        B = len(kvs)
        arr = (P * B)(*[k._h for k in kvs])
        out = np.empty((B, self.vocab), dtype=np.float32)
        st = lib().or_decode_batch(self._h, arr, B, ids.ctypes.data, out.ctypes.data)
        if st:
            raise ValueError(f"or_decode_batch status {st}")
        return out


class KV:
    def __init__(self, model: Model, max_ctx: int):
        self._h = lib().or_kv_new(model._h, max_ctx)
        self.model = model

    def __len__(self):
        return lib().or_kv_len(self._h)

    def fill_synthetic(self, n: int, seed: int = 0):
        st = lib().or_kv_fill_synthetic(self._h, n, seed)
        if st:
            raise ValueError("kv fill failed")

    def close(self):
        if self._h:
            lib().or_kv_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
