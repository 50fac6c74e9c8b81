"""Device ops with the reference's op signatures, on torch CUDA tensors.

torch only provides device memory and the current stream here; every op runs
a kernel of libwoolly_cuda.so and raises if the library or the GPU is missing.
"""
from __future__ import annotations

import numpy as np
import torch

from ._lib import LAYOUT_A, LAYOUT_B, ROPE_NEOX, ROPE_OFF, check, lib


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dev(t: torch.Tensor, dtype=None, name="tensor") -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return t


def dequantize(data: torch.Tensor, ggml_type: int, nelements: int) -> torch.Tensor:
    """woolly_gguf::dequantize(data, ggml_type, nelements) (dequantize.rs:189)."""
    _dev(data, torch.uint8, "data")
    out = torch.empty(nelements, dtype=torch.float32, device=data.device)
    check(lib().wl_dequantize(int(ggml_type), data.data_ptr(), data.numel(), nelements,
                              out.data_ptr(), _stream()))
    return out


def quantized_matvec(weights: torch.Tensor, ggml_type: int, input: torch.Tensor,
                     output: torch.Tensor, m: int, k: int) -> None:
    """quantization::simd::quantized_matvec(weights, input, output, m, k)
    (woolly-tensor/src/quantization.rs:869): layout A, Q4_0 / Q8_0."""
    _dev(weights, torch.uint8, "weights")
    _dev(input, torch.float32, "input")
    _dev(output, torch.float32, "output")
    if input.numel() < k or output.numel() < m:
        raise ValueError("input/output too small")
    check(lib().wl_quantized_matvec(int(ggml_type), weights.data_ptr(), input.data_ptr(),
                                    output.data_ptr(), m, k, _stream()))


def qgemv(weights: torch.Tensor, ggml_type: int, layout: int, x: torch.Tensor, n: int) -> torch.Tensor:
    """y[b, :] = x[b, :] @ W for quantized W ([K][N] layout B or [N][K] layout A)."""
    _dev(weights, torch.uint8, "weights")
    _dev(x, torch.float32, "x")
    x2 = x.reshape(-1, x.shape[-1])
    B, K = x2.shape
    y = torch.empty(B, n, dtype=torch.float32, device=x.device)
    check(lib().wl_qgemv(int(ggml_type), int(layout), weights.data_ptr(), K, n, x2.data_ptr(), B,
                         y.data_ptr(), _stream()))
    return y.reshape(*x.shape[:-1], n)


def qgemm(weights: torch.Tensor, ggml_type: int, x: torch.Tensor, n: int) -> torch.Tensor:
    """Prefill GEMM y[m, :] = x[m, :] @ W for layout-B W ([K][N] GGUF blocks),
    all rows in one call (tcgen05 tensor cores where the shape allows)."""
    _dev(weights, torch.uint8, "weights")
    _dev(x, torch.float32, "x")
    x2 = x.reshape(-1, x.shape[-1])
    M, K = x2.shape
    y = torch.empty(M, n, dtype=torch.float32, device=x.device)
    check(lib().wl_qgemm(int(ggml_type), weights.data_ptr(), K, n, x2.data_ptr(), M, y.data_ptr(),
                         _stream()))
    return y.reshape(*x.shape[:-1], n)


def split_planes(x: torch.Tensor) -> torch.Tensor:
    """f32 [B, K] -> f16 [2, B, K]: hi = f16(x), lo = f16(x - hi)."""
    hi = x.to(torch.float16)
    return torch.stack([hi, (x - hi.float()).to(torch.float16)]).contiguous()


def qgemv_planes(weights: torch.Tensor, ggml_type: int, planes: torch.Tensor, n: int,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Layout-B GEMV on hi/lo activation planes [2, B, K] (no allocation
    inside the library; capturable in a CUDA graph)."""
    _dev(weights, torch.uint8, "weights")
    _dev(planes, torch.float16, "planes")
    _, B, K = planes.shape
    y = out if out is not None else torch.empty(B, n, dtype=torch.float32, device=planes.device)
    check(lib().wl_qgemv_planes(int(ggml_type), weights.data_ptr(), K, n, planes.data_ptr(), B * K,
                                B, y.data_ptr(), _stream()))
    return y


def qtile(weights: torch.Tensor, ggml_type: int, k: int, n: int) -> torch.Tensor:
    """Tiled decode copy of a layout-B GGUF matrix [k][n] (wl_qtile_repack)."""
    _dev(weights, torch.uint8, "weights")
    nb = lib().wl_qtile_bytes(int(ggml_type), k, n)
    if not nb:
        raise ValueError(f"qtile: unsupported type {ggml_type} or shape {k}x{n}")
    t = torch.empty(nb, dtype=torch.uint8, device=weights.device)
    check(lib().wl_qtile_repack(int(ggml_type), weights.data_ptr(), k, n, t.data_ptr(), _stream()))
    return t


def qgemv_tiled(tiled: torch.Tensor, ggml_type: int, planes: torch.Tensor, n: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """qgemv_planes on the tiled copy made by qtile()."""
    _dev(tiled, torch.uint8, "tiled")
    _dev(planes, torch.float16, "planes")
    _, B, K = planes.shape
    y = out if out is not None else torch.empty(B, n, dtype=torch.float32, device=planes.device)
    check(lib().wl_qgemv_tiled(int(ggml_type), tiled.data_ptr(), K, n, planes.data_ptr(), B * K,
                               B, y.data_ptr(), _stream()))
    return y


def qgemm_tiled(tiled: torch.Tensor, ggml_type: int, planes: torch.Tensor, n: int,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """The tcgen05 prefill GEMM on the tiled copy made by qtile(); planes [2, M, K]."""
    _dev(tiled, torch.uint8, "tiled")
    _dev(planes, torch.float16, "planes")
    _, M, K = planes.shape
    y = out if out is not None else torch.empty(M, n, dtype=torch.float32, device=planes.device)
    check(lib().wl_qgemm_tiled(int(ggml_type), tiled.data_ptr(), K, n, planes.data_ptr(), M * K, M,
                               y.data_ptr(), _stream()))
    return y


def rmsnorm_rope(x: torch.Tensor, w: torch.Tensor, eps: float, *, rope: bool = False,
                 positions: torch.Tensor | None = None, head_dim: int = 0, theta: float = 10000.0,
                 out_dtype=torch.float32) -> torch.Tensor:
    """rms_norm (woolly-core tensor_utils.rs:446-480) with an optional fused NeoX
    RoPE of the normalised row (woolly-tensor ops/mod.rs:476-527)."""
    _dev(x, torch.float32, "x")
    _dev(w, torch.float32, "w")
    d = x.shape[-1]
    rows = x.numel() // d
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    pos_ptr = None
    if rope:
        if positions is None:
            raise ValueError("rope needs positions")
        _dev(positions, torch.int32, "positions")
        pos_ptr = positions.data_ptr()
    check(lib().wl_rmsnorm_rope(x.data_ptr(), w.data_ptr(), rows, d, eps,
                                ROPE_NEOX if rope else ROPE_OFF, pos_ptr, head_dim, theta,
                                y.data_ptr(), 1 if out_dtype == torch.float16 else 0, _stream()))
    return y


class TransformerSIMD:
    """woolly_tensor::ops::simd_matmul::TransformerSIMD (simd_matmul.rs:811,1002)."""

    @staticmethod
    def rms_norm(input: torch.Tensor, weight: torch.Tensor, eps: float, output: torch.Tensor) -> None:
        d = weight.numel()
        _dev(output, torch.float32, "output")
        y = rmsnorm_rope(input.reshape(-1, d), weight, eps)
        output.copy_(y.reshape(output.shape))

    @staticmethod
    def swiglu_activation(gate: torch.Tensor, up: torch.Tensor, output: torch.Tensor) -> None:
        _dev(gate, torch.float32, "gate")
        _dev(up, torch.float32, "up")
        _dev(output, torch.float32, "output")
        if gate.numel() != up.numel() or output.numel() != gate.numel():
            raise ValueError("gate, up and output must have the same length")
        check(lib().wl_swiglu(gate.data_ptr(), up.data_ptr(), gate.numel(), output.data_ptr(),
                              _stream()))


class RoPE:
    """woolly_tensor::ops::neural::RoPE (ops/mod.rs:472-527)."""

    @staticmethod
    def apply_f32(input: torch.Tensor, output: torch.Tensor, positions: torch.Tensor, base: float,
                  batch_size: int, seq_len: int, n_heads: int, head_dim: int) -> None:
        _dev(input, torch.float32, "input")
        _dev(output, torch.float32, "output")
        _dev(positions, torch.int32, "positions")
        if input.numel() != batch_size * seq_len * n_heads * head_dim:
            raise ValueError("input size mismatch")
        if positions.numel() != seq_len:
            raise ValueError("positions must have seq_len entries")
        check(lib().wl_rope(input.data_ptr(), output.data_ptr(), positions.data_ptr(), base,
                            batch_size, seq_len, n_heads, head_dim, _stream()))


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, past: int, heads: int,
              kv_heads: int, head_dim: int, window: int = 0) -> torch.Tensor:
    """GQA attention over an f32 KV prefix (lazy_transformer.rs:375-434):
    q [rows, H*hd], k/v [past+rows, KVH*hd]."""
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _dev(t, torch.float32, n)
    rows = q.numel() // (heads * head_dim)
    out = torch.empty(rows, heads * head_dim, dtype=torch.float32, device=q.device)
    check(lib().wl_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), rows, past, heads, kv_heads,
                             head_dim, window, out.data_ptr(), _stream()))
    return out


__all__ = ["dequantize", "quantized_matvec", "qgemv", "rmsnorm_rope", "TransformerSIMD", "RoPE",
           "attention", "LAYOUT_A", "LAYOUT_B"]


def sample(logits: torch.Tensor, temperature, top_k, top_p, u, out: torch.Tensor | None = None,
           params: torch.Tensor | None = None) -> torch.Tensor:
    """sample_next_token (inference.rs:441-483) for every row of f32 logits
    [rows, vocab] on the GPU; temperature / top_k / top_p / u are per-row
    sequences (or scalars).  `params` (optional): a device buffer of at least
    rows * 16 bytes to stage them in.  Returns int32 token ids [rows]."""
    _dev(logits, torch.float32, "logits")
    rows, V = logits.shape
    rec = sample_params(rows, temperature, top_k, top_p, u)
    src = torch.from_numpy(rec.view(np.uint8))
    if params is None:
        params = src.to(logits.device)
    else:
        params[: src.numel()].copy_(src)
    y = out if out is not None else torch.empty(rows, dtype=torch.int32, device=logits.device)
    check(lib().wl_sample(logits.data_ptr(), rows, V, logits.stride(0), params.data_ptr(),
                          y.data_ptr(), _stream()))
    return y


def sample_params(rows, temperature, top_k, top_p, u) -> "np.ndarray":
    """Per-row knobs as an array of wl_sample_params records."""
    rec = np.zeros(rows, dtype=[("t", "<f4"), ("k", "<i4"), ("p", "<f4"), ("u", "<f4")])
    rec["t"], rec["k"], rec["p"], rec["u"] = temperature, top_k, top_p, u
    return rec
