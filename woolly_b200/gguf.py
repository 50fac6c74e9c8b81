"""GGUF access mirroring woolly-gguf's public surface (GGUFLoader, TensorInfo,
GGMLType), backed by the C++ parser in libwoolly_cuda.so.

Reference: crates/woolly-gguf/src/{loader.rs,tensor_info.rs,format.rs,metadata.rs}.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from enum import IntEnum

import numpy as np

from . import _lib
from ._lib import check, lib


class GGMLType(IntEnum):
    """GGMLType (crates/woolly-gguf/src/tensor_info.rs:15-73)."""
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q8_1 = 9
    Q2_K = 10
    Q3_K = 11
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    Q8_K = 15
    I8 = 24
    I16 = 25
    I32 = 26
    I64 = 27
    F64 = 28
    BF16 = 30

    def block_size(self) -> int:
        return int(lib().wl_block_size(int(self)))

    def type_size(self) -> int:
        return int(lib().wl_type_size(int(self)))

    def is_quantized(self) -> bool:
        return self not in (GGMLType.F32, GGMLType.F16, GGMLType.BF16, GGMLType.F64,
                            GGMLType.I8, GGMLType.I16, GGMLType.I32, GGMLType.I64)


@dataclass
class TensorInfo:
    name: str
    shape: tuple
    ggml_type: int
    offset: int
    data_size: int

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n


@dataclass
class GGUFHeader:
    version: int
    tensor_count: int
    metadata_kv_count: int


class GGUFLoader:
    """GGUFLoader::from_path (loader.rs:112).  Errors raise WoollyError with
    the reference's error kinds (InvalidMagic, UnsupportedVersion, Io, ...)."""

    def __init__(self, handle: C.c_void_p, keepalive=None):
        self._h = handle
        self._keep = keepalive

    @classmethod
    def from_path(cls, path: str) -> "GGUFLoader":
        h = C.c_void_p()
        check(lib().wl_gguf_open(str(path).encode(), C.byref(h)))
        return cls(h)

    @classmethod
    def from_bytes(cls, data: bytes) -> "GGUFLoader":
        h = C.c_void_p()
        buf = C.create_string_buffer(bytes(data), len(data)) if data else None
        check(lib().wl_gguf_open_memory(buf, len(data), C.byref(h)))
        return cls(h)

    def close(self) -> None:
        if self._h:
            lib().wl_gguf_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def header(self) -> GGUFHeader:
        v, tc, kc, al, ds = C.c_uint32(), C.c_uint64(), C.c_uint64(), C.c_uint32(), C.c_uint64()
        check(lib().wl_gguf_header(self._h, C.byref(v), C.byref(tc), C.byref(kc), C.byref(al),
                                   C.byref(ds)))
        return GGUFHeader(v.value, tc.value, kc.value)

    def alignment(self) -> int:
        al = C.c_uint32()
        check(lib().wl_gguf_header(self._h, None, None, None, C.byref(al), None))
        return al.value

    def data_start(self) -> int:
        ds = C.c_uint64()
        check(lib().wl_gguf_header(self._h, None, None, None, None, C.byref(ds)))
        return ds.value

    def _info(self, ti: _lib.TensorInfo) -> TensorInfo:
        return TensorInfo(ti.name.decode(), tuple(ti.dims[i] for i in range(ti.n_dims)),
                          int(ti.ggml_type), int(ti.offset), int(ti.nbytes))

    def tensors(self) -> list[TensorInfo]:
        out = []
        for i in range(lib().wl_gguf_tensor_count(self._h)):
            ti = _lib.TensorInfo()
            check(lib().wl_gguf_tensor(self._h, i, C.byref(ti)))
            out.append(self._info(ti))
        return out

    def tensor_names(self) -> list[str]:
        return [t.name for t in self.tensors()]

    def tensor_info(self, name: str) -> TensorInfo:
        ti = _lib.TensorInfo()
        check(lib().wl_gguf_find_tensor(self._h, name.encode(), C.byref(ti)))
        return self._info(ti)

    def tensor_data(self, name: str) -> np.ndarray:
        """Raw tensor bytes (uint8 copy), loader.rs:230-295."""
        p, n = C.c_void_p(), C.c_uint64()
        check(lib().wl_gguf_tensor_data(self._h, name.encode(), C.byref(p), C.byref(n)))
        return np.ctypeslib.as_array((C.c_uint8 * n.value).from_address(p.value)).copy()

    def get_u32(self, key: str):
        v = C.c_uint32()
        return v.value if lib().wl_gguf_get_u32(self._h, key.encode(), C.byref(v)) == 0 else None

    def get_f32(self, key: str):
        v = C.c_float()
        return v.value if lib().wl_gguf_get_f32(self._h, key.encode(), C.byref(v)) == 0 else None

    def get_str(self, key: str):
        p, n = C.c_char_p(), C.c_uint64()
        if lib().wl_gguf_get_str(self._h, key.encode(), C.byref(p), C.byref(n)) != 0:
            return None
        return C.string_at(p, n.value).decode()

    def architecture(self):
        return self.get_str("general.architecture")

    def model_config(self) -> dict:
        """GGUFModelLoader::extract_config (woolly-core/src/model/loader.rs:104-156)."""
        c = _lib.ModelConfig()
        check(lib().wl_gguf_model_config(self._h, C.byref(c)))
        return config_dict(c)


def config_dict(c: _lib.ModelConfig) -> dict:
    return {
        "architecture": c.architecture.decode(),
        "vocab_size": c.vocab_size,
        "hidden_size": c.hidden_size,
        "num_layers": c.num_layers,
        "num_heads": c.num_heads,
        "context_length": c.context_length,
        "intermediate_size": c.intermediate_size,
        "num_key_value_heads": c.num_kv_heads_meta or None,
        "rope_theta": c.rope_theta or None,
        "layer_norm_epsilon": c.layer_norm_epsilon,
    }


def write_synthetic(path: str, *, hidden: int, layers: int, heads: int, kv_heads: int, ff: int,
                    vocab: int, weight_type: int = _lib.Q4_0, output_type: int | None = None,
                    tied: bool = False, context_length: int = 4096, sliding_window: int = 0,
                    rope_theta: float = 10000.0, norm_eps: float = 1e-5, seed: int = 0,
                    vd_type: int = 0, embd_type: int = 0) -> str:
    """Writes the seeded LLaMA-shape GGUF used by the tests and benchmarks.
    vd_type (0 = weight_type) is the type of attn_v and ffn_down, as the
    K-quant mixes store them (Q6_K beside Q4_K); embd_type that of
    token_embd.weight (F32 by default)."""
    cfg = _lib.SynthConfig(hidden, layers, heads, kv_heads, ff, vocab, context_length,
                           weight_type,
                           0xFFFFFFFF if tied else (weight_type if output_type is None
                                                    else output_type),
                           sliding_window, rope_theta, norm_eps, seed, vd_type, embd_type)
    check(lib().wl_synth_gguf(str(path).encode(), C.byref(cfg)))
    return str(path)


def quantize(ggml_type: int, values: np.ndarray) -> np.ndarray:
    """Encodes f32 values (len % 32 == 0) into GGUF blocks."""
    v = np.ascontiguousarray(values, dtype=np.float32).ravel()
    nb = v.size // int(lib().wl_block_size(ggml_type)) * int(lib().wl_type_size(ggml_type))
    out = np.zeros(nb, dtype=np.uint8)
    check(lib().wl_quantize(ggml_type, v.ctypes.data, v.size, out.ctypes.data))
    return out


def synth_normal(seed: int, stream: int, n: int, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    check(lib().wl_synth_normal(seed, stream, mean, std, n, out.ctypes.data))
    return out
