"""ctypes binding of libwoolly_cuda.so (the C ABI in include/woolly_cuda.h).

The library is loaded from this package directory; there is no fallback: if
it is missing, importing the compute entry points raises.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libwoolly_cuda.so")

# wl_status codes
WL_OK = 0
WL_ERR_INVALID_ARGUMENT = 1
WL_ERR_IO = 2
WL_ERR_INVALID_MAGIC = 3
WL_ERR_UNSUPPORTED_VERSION = 4
WL_ERR_INVALID_FORMAT = 5
WL_ERR_INVALID_TENSOR_TYPE = 6
WL_ERR_BUFFER_TOO_SMALL = 7
WL_ERR_TENSOR_NOT_FOUND = 8
WL_ERR_UNSUPPORTED = 9
WL_ERR_CUDA = 10
WL_ERR_OUT_OF_MEMORY = 11
WL_ERR_CONTEXT_FULL = 12
WL_ERR_TOKEN_OUT_OF_RANGE = 13
WL_ERR_NCCL = 14
WL_ERR_TIMEOUT = 15

F32, F16, Q4_0, Q4_1, Q8_0 = 0, 1, 2, 3, 8
Q4_K, Q6_K = 12, 14
LAYOUT_A, LAYOUT_B = 0, 1
ROPE_OFF, ROPE_NEOX = 0, 1
LOGITS_LAST, LOGITS_ALL = 0, 1


class WoollyError(RuntimeError):
    """A failed wl_* call: `.code` is the wl_status, the message is wl_last_error()."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


class TensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4),
                ("ggml_type", C.c_uint32), ("offset", C.c_uint64), ("nbytes", C.c_uint64)]


class ModelConfig(C.Structure):
    _fields_ = [("vocab_size", C.c_uint32), ("hidden_size", C.c_uint32),
                ("num_layers", C.c_uint32), ("num_heads", C.c_uint32),
                ("context_length", C.c_uint32), ("intermediate_size", C.c_uint32),
                ("num_kv_heads_meta", C.c_uint32), ("rope_theta", C.c_float),
                ("layer_norm_epsilon", C.c_float), ("architecture", C.c_char * 64)]


class SampleParams(C.Structure):
    """wl_sample_params: one row's sampling knobs and uniform draw."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int), ("top_p", C.c_float),
                ("u", C.c_float)]


class SynthConfig(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("layers", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("ff", C.c_uint32), ("vocab", C.c_uint32),
                ("context_length", C.c_uint32), ("weight_type", C.c_uint32),
                ("output_type", C.c_uint32), ("sliding_window", C.c_uint32),
                ("rope_theta", C.c_float), ("norm_eps", C.c_float), ("seed", C.c_uint64),
                ("vd_type", C.c_uint32), ("embd_type", C.c_uint32)]


class ModelOptions(C.Structure):
    _fields_ = [("rope_mode", C.c_int), ("sliding_window", C.c_int), ("max_sessions", C.c_int),
                ("max_context", C.c_int), ("max_batch", C.c_int), ("max_prefill", C.c_int),
                ("use_graphs", C.c_int), ("tp_rank", C.c_int), ("tp_size", C.c_int),
                ("nccl_comm", C.c_void_p), ("ggml_layout", C.c_int),
                ("collective_timeout_ms", C.c_int)]


P = C.c_void_p
_SIGS = {
    "wl_last_error": (C.c_char_p, []),
    "wl_version": (C.c_char_p, []),
    "wl_block_size": (C.c_size_t, [C.c_int]),
    "wl_type_size": (C.c_size_t, [C.c_int]),
    "wl_gguf_open": (C.c_int, [C.c_char_p, C.POINTER(P)]),
    "wl_gguf_open_memory": (C.c_int, [P, C.c_size_t, C.POINTER(P)]),
    "wl_gguf_close": (None, [P]),
    "wl_gguf_header": (C.c_int, [P, C.POINTER(C.c_uint32), C.POINTER(C.c_uint64),
                                 C.POINTER(C.c_uint64), C.POINTER(C.c_uint32),
                                 C.POINTER(C.c_uint64)]),
    "wl_gguf_tensor_count": (C.c_int, [P]),
    "wl_gguf_tensor": (C.c_int, [P, C.c_int, C.POINTER(TensorInfo)]),
    "wl_gguf_find_tensor": (C.c_int, [P, C.c_char_p, C.POINTER(TensorInfo)]),
    "wl_gguf_tensor_data": (C.c_int, [P, C.c_char_p, C.POINTER(P), C.POINTER(C.c_uint64)]),
    "wl_gguf_model_config": (C.c_int, [P, C.POINTER(ModelConfig)]),
    "wl_gguf_get_u32": (C.c_int, [P, C.c_char_p, C.POINTER(C.c_uint32)]),
    "wl_gguf_get_f32": (C.c_int, [P, C.c_char_p, C.POINTER(C.c_float)]),
    "wl_gguf_get_str": (C.c_int, [P, C.c_char_p, C.POINTER(C.c_char_p), C.POINTER(C.c_uint64)]),
    "wl_synth_gguf": (C.c_int, [C.c_char_p, C.POINTER(SynthConfig)]),
    "wl_quantize": (C.c_int, [C.c_int, P, C.c_size_t, P]),
    "wl_synth_normal": (C.c_int, [C.c_uint64, C.c_uint64, C.c_float, C.c_float, C.c_size_t, P]),
    "wl_dequantize": (C.c_int, [C.c_int, P, C.c_size_t, C.c_size_t, P, P]),
    "wl_qgemv": (C.c_int, [C.c_int, C.c_int, P, C.c_int, C.c_int, P, C.c_int, P, P]),
    "wl_qgemv_planes": (C.c_int, [C.c_int, P, C.c_int, C.c_int, P, C.c_size_t, C.c_int, P, P]),
    "wl_qtile_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
    "wl_qtile_repack": (C.c_int, [C.c_int, P, C.c_int, C.c_int, P, P]),
    "wl_qgemv_tiled": (C.c_int, [C.c_int, P, C.c_int, C.c_int, P, C.c_size_t, C.c_int, P, P]),
    "wl_qgemm_tiled": (C.c_int, [C.c_int, P, C.c_int, C.c_int, P, C.c_size_t, C.c_int, P, P]),
    "wl_qgemv_noalloc": (C.c_int, [C.c_int, P, C.c_int, C.c_int, P, C.c_int, P, P]),
    "wl_quantized_matvec": (C.c_int, [C.c_int, P, P, P, C.c_int, C.c_int, P]),
    "wl_rmsnorm_rope": (C.c_int, [P, P, C.c_int, C.c_int, C.c_float, C.c_int, P, C.c_int,
                                  C.c_float, P, C.c_int, P]),
    "wl_tp_reduce_rmsnorm": (C.c_int, [P, P, C.c_int, C.c_int, C.c_float, P, C.c_int, P, C.c_uint,
                                       P, C.c_size_t, P, P]),
    "wl_swiglu": (C.c_int, [P, P, C.c_size_t, P, P]),
    "wl_nccl_comm_abort": (C.c_int, [P]),
    "wl_sample": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, P, P]),
    "wl_rope": (C.c_int, [P, P, P, C.c_float, C.c_int, C.c_int, C.c_int, C.c_int, P]),
    "wl_attention": (C.c_int, [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                               P, P]),
    "wl_model_options_default": (None, [C.POINTER(ModelOptions)]),
    "wl_init": (C.c_int, [C.c_int, C.POINTER(P)]),
    "wl_ctx_free": (None, [P]),
    "wl_model_load_gguf": (C.c_int, [P, C.c_char_p, C.POINTER(ModelOptions), C.POINTER(P)]),
    "wl_model_free": (None, [P]),
    "wl_model_get_config": (C.c_int, [P, C.POINTER(ModelConfig)]),
    "wl_model_memory": (C.c_int, [P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "wl_session_create": (C.c_int, [P, C.POINTER(P)]),
    "wl_session_free": (None, [P]),
    "wl_session_reset": (C.c_int, [P]),
    "wl_session_length": (C.c_int, [P]),
    "wl_forward": (C.c_int, [P, C.POINTER(P), C.c_int, P, P, P, C.c_int]),
    "wl_decode_step_device": (C.c_int, [P, C.POINTER(P), C.c_int, P, P, P]),
    "wl_decode_kernel_count": (C.c_int, [P, C.c_int]),
    "wl_qgemm": (C.c_int, [C.c_int, P, C.c_int, C.c_int, P, C.c_int, P, P]),
    "wl_nccl_unique_id": (C.c_int, [P]),
    "wl_nccl_comm_init": (C.c_int, [C.c_int, P, C.c_int, C.POINTER(P)]),
    "wl_nccl_comm_destroy": (C.c_int, [P]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads libwoolly_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m woolly_b200.build`")
        h = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(status: int) -> None:
    if status != WL_OK:
        msg = lib().wl_last_error()
        raise WoollyError(status, msg.decode() if msg else "")
