"""Op-level parity of the CUDA kernels against the CPU oracle (GPU).

Tolerances: dequantization is bit-exact (integer unpack and f16 widening
must match woolly_gguf::dequantize exactly).  The GEMV feeds the tensor cores
f16 operands (weights rounded once to f16, activations rounded to f16) and
accumulates in f32: |y - ref| <= 4e-3 * max|ref| per output vector.  f32 ops
(RMSNorm, SwiGLU, RoPE, attention) are held to 2e-5 relative.
"""
import json
import os
import struct

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from woolly_b200 import LAYOUT_A, LAYOUT_B, Q4_0, Q4_1, Q8_0, WoollyError, _lib  # noqa: E402
from woolly_b200 import ops  # noqa: E402
from woolly_b200.gguf import quantize  # noqa: E402

GOLD = os.path.join(os.path.dirname(__file__), "golden")
TS = {Q4_0: 18, Q4_1: 20, Q8_0: 34}
GEMV_TOL = 4e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def random_blocks(qt, nb, seed, scales=(0.0123, -0.5, 3e-5, 1.0, 6e-8, 2.0)):
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(nb, TS[qt]), dtype=np.uint8)
    sc = rng.choice(np.array(scales, np.float16), nb * 2)
    raw[:, 0:2] = sc[:nb].view(np.uint8).reshape(nb, 2)
    if qt == Q4_1:
        raw[:, 2:4] = sc[nb:].view(np.uint8).reshape(nb, 2)
    return raw.reshape(-1)


def quant_matrix(qt, rows, cols, seed, std=0.02):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(rows * cols) * std).astype(np.float32)
    return quantize(qt, w)


@pytest.mark.parametrize("qt", [Q4_0, Q4_1, Q8_0])
def test_dequant_bit_exact(qt):
    nb = 50_000
    raw = random_blocks(qt, nb, qt)
    ref = O.dequantize(raw.tobytes(), qt, nb * 32)
    got = ops.dequantize(dev(raw), qt, nb * 32).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("qt", [Q4_0, Q4_1, Q8_0])
def test_dequant_any_bytes_and_partial_block(qt):
    nb = 4096
    raw = np.random.default_rng(100 + qt).integers(0, 256, size=nb * TS[qt], dtype=np.uint8)
    n = nb * 32 - 7
    ref = O.dequantize(raw.tobytes(), qt, n)
    got = ops.dequantize(dev(raw), qt, n).cpu().numpy()
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_dequant_kats_on_gpu():
    with open(os.path.join(GOLD, "kats.json")) as f:
        kats = json.load(f)["dequant"]
    for k in kats:
        raw = np.frombuffer(bytes.fromhex(k["hex"]), np.uint8)
        got = ops.dequantize(dev(raw), k["type"], k["n"]).cpu().numpy()
        assert got.tolist() == k["expect"], k["source"]


def test_dequant_buffer_too_small():
    with pytest.raises(WoollyError) as e:
        ops.dequantize(dev(np.zeros(17, np.uint8)), Q4_0, 32)
    assert e.value.code == _lib.WL_ERR_BUFFER_TOO_SMALL


def ref_gemv(qt, layout, raw, K, N, x):
    W = O.dequantize(raw.tobytes(), qt, K * N).astype(np.float64)
    W = W.reshape(K, N) if layout == LAYOUT_B else W.reshape(N, K).T
    return x.astype(np.float64) @ W


def check_gemv(y, ref):
    y = np.asarray(y, np.float64)
    scale = np.abs(ref).max()
    assert np.abs(y - ref).max() <= GEMV_TOL * scale + 1e-6, (np.abs(y - ref).max(), scale)


@pytest.mark.parametrize("qt", [Q4_0, Q4_1, Q8_0])
@pytest.mark.parametrize("layout", [LAYOUT_B, LAYOUT_A])
@pytest.mark.parametrize("K,N", [(512, 1024), (2048, 256), (768, 96), (256, 4096), (160, 64)])
@pytest.mark.parametrize("B", [1, 3, 5, 16, 33])
def test_qgemv_vs_oracle(qt, layout, K, N, B):
    raw = quant_matrix(qt, K, N, seed=K * 7 + N + qt)
    x = np.random.default_rng(B).standard_normal((B, K)).astype(np.float32)
    y = ops.qgemv(dev(raw), qt, layout, dev(x), N).cpu().numpy()
    check_gemv(y, ref_gemv(qt, layout, raw, K, N, x))


@pytest.mark.parametrize("qt", [Q4_0, Q4_1, Q8_0])
@pytest.mark.parametrize("K,N", [(4096, 4096), (4096, 14336), (14336, 4096)])
def test_qgemv_sweep_shapes(qt, K, N):
    """The standalone sweep shapes, both layouts, B = 1 and 16."""
    raw = quant_matrix(qt, K, N, seed=3)
    W = O.dequantize(raw.tobytes(), qt, K * N).astype(np.float32)
    for layout in (LAYOUT_B, LAYOUT_A):
        Wm = W.reshape(K, N) if layout == LAYOUT_B else W.reshape(N, K).T
        Wt = dev(Wm)
        for B in (1, 16):
            x = np.random.default_rng(B).standard_normal((B, K)).astype(np.float32)
            y = ops.qgemv(dev(raw), qt, layout, dev(x), N)
            ref = (dev(x).double() @ Wt.double()).cpu().numpy()
            check_gemv(y.cpu().numpy(), ref)


@pytest.mark.parametrize("qt", [Q4_0, Q4_1, Q8_0])
def test_qgemv_planes_matches_f32_entry(qt):
    K, N, B = 1024, 768, 20
    raw = quant_matrix(qt, K, N, seed=77)
    x = dev(np.random.default_rng(5).standard_normal((B, K)).astype(np.float32))
    ref = ops.qgemv(dev(raw), qt, LAYOUT_B, x, N)
    got = ops.qgemv_planes(dev(raw), qt, ops.split_planes(x), N)
    assert torch.equal(ref, got)


@pytest.mark.parametrize("qt", [Q4_0, Q4_1, Q8_0])
@pytest.mark.parametrize("K,N", [(512, 1024), (80, 288), (768, 96), (4096, 4096), (11008, 4096)])
@pytest.mark.parametrize("B", [1, 3, 5, 16, 33])
def test_qgemv_tiled_vs_oracle(qt, K, N, B):
    """The tiled decode copy (ragged last group N = 288, a partial last stage
    K = 80, LOC for B <= 4) against the restatement, and within f32 summation
    order of the GGUF-layout kernel on the same planes where that kernel takes
    the shape (16-byte rows; the repack reads any row pitch)."""
    raw = quant_matrix(qt, K, N, seed=K + N + qt)
    x = np.random.default_rng(B + 11).standard_normal((B, K)).astype(np.float32)
    planes = ops.split_planes(dev(x))
    W = dev(raw)
    tiled = ops.qtile(W, qt, K, N)
    assert tiled.numel() == (N + 255) // 256 * ((K + 63) // 64) * 512 * TS[qt]
    y = ops.qgemv_tiled(tiled, qt, planes, N)
    ref = ref_gemv(qt, LAYOUT_B, raw, K, N, x)
    check_gemv(y.cpu().numpy(), ref)
    if (N // 32 * TS[qt]) % 16:
        return
    y0 = ops.qgemv_planes(W, qt, planes, N)
    assert (y - y0).abs().max().item() <= 1e-5 * max(1.0, float(np.abs(ref).max()))


def test_qtile_rejects_bad_shapes():
    assert _lib.lib().wl_qtile_bytes(Q4_0, 64, 48) == 0
    assert _lib.lib().wl_qtile_bytes(12, 64, 64) == 0
    W = torch.zeros(64 * 2 * 18, dtype=torch.uint8, device="cuda")
    with pytest.raises((ValueError, WoollyError)):
        ops.qtile(W, Q4_0, 64, 48)


def test_matmul_2x2_kat_layout_b():
    """tensor_utils.rs:608-620 ([1,2;3,4] @ [5,6;7,8] = [19,22;43,50]) through the
    layout-B GEMV with Q8_0 blocks of scale 1: the K=2 case takes the generic
    kernel, the zero-padded K=32 case the tensor-core kernel."""
    for K in (2, 32):
        Wf = np.zeros((K, 32), np.float32)
        Wf[0, :2] = [5, 6]
        Wf[1, :2] = [7, 8]
        raw = bytearray()
        for r in range(K):
            raw += struct.pack("<e", 1.0) + Wf[r].astype(np.int8).tobytes()
        x = np.zeros((2, K), np.float32)
        x[0, :2] = [1, 2]
        x[1, :2] = [3, 4]
        y = ops.qgemv(dev(np.frombuffer(bytes(raw), np.uint8)), Q8_0, LAYOUT_B, dev(x), 32)
        assert y[:, :2].cpu().numpy().ravel().tolist() == [19.0, 22.0, 43.0, 50.0]


@pytest.mark.parametrize("qt", [Q4_0, Q8_0])
def test_quantized_matvec_vs_scalar_reference(qt):
    m, k = 1024, 4096
    raw = quant_matrix(qt, m, k, seed=9)
    x = np.random.default_rng(1).standard_normal(k).astype(np.float32)
    ref = O.quantized_matvec(qt, raw, x, m, k).astype(np.float64)
    out = torch.zeros(m, dtype=torch.float32, device="cuda")
    ops.quantized_matvec(dev(raw), qt, dev(x), out, m, k)
    check_gemv(out.cpu().numpy(), ref)


def test_quantized_matvec_q4_1_unsupported():
    out = torch.zeros(1, dtype=torch.float32, device="cuda")
    with pytest.raises(WoollyError) as e:
        ops.quantized_matvec(dev(np.zeros(40, np.uint8)), Q4_1, dev(np.zeros(64, np.float32)), out, 1, 64)
    assert e.value.code == _lib.WL_ERR_UNSUPPORTED


@pytest.mark.parametrize("d", [64, 1030, 2048, 4096, 5120, 12288, 16384])
def test_rmsnorm(d):
    rng = np.random.default_rng(d)
    x = rng.standard_normal((7, d)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(d)).astype(np.float32)
    ref = O.rms_norm(x, w, 1e-5)
    y = ops.rmsnorm_rope(dev(x), dev(w), 1e-5).cpu().numpy()
    assert np.allclose(y, ref, rtol=2e-5, atol=1e-6)
    yh = ops.rmsnorm_rope(dev(x), dev(w), 1e-5, out_dtype=torch.float16).cpu().numpy()
    assert np.allclose(yh.astype(np.float32), ref.astype(np.float16).astype(np.float32),
                       rtol=1e-3, atol=1e-3)


def test_rmsnorm_fused_rope():
    rng = np.random.default_rng(5)
    rows, heads, hd = 6, 8, 64
    x = rng.standard_normal((rows, heads * hd)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(heads * hd)).astype(np.float32)
    pos = np.array([0, 1, 7, 100, 1000, 4095], np.int32)
    normed = O.rms_norm(x, w, 1e-5)
    ref = np.stack([O.rope_neox(normed[r], [pos[r]], 1, 1, heads, hd, 10000.0) for r in range(rows)])
    y = ops.rmsnorm_rope(dev(x), dev(w), 1e-5, rope=True, positions=dev(pos), head_dim=hd).cpu().numpy()
    assert np.allclose(y, ref.reshape(rows, -1), rtol=5e-5, atol=5e-5)


def test_swiglu_exact():
    rng = np.random.default_rng(2)
    g = (rng.standard_normal(100_003) * 4).astype(np.float32)
    u = rng.standard_normal(100_003).astype(np.float32)
    ref = O.swiglu(g, u, 0)
    out = torch.empty(g.size, dtype=torch.float32, device="cuda")
    ops.TransformerSIMD.swiglu_activation(dev(g), dev(u), out)
    assert np.allclose(out.cpu().numpy(), ref, rtol=2e-6, atol=1e-7)


def test_rope_apply_f32():
    rng = np.random.default_rng(3)
    batch, seq, heads, hd = 2, 5, 4, 128
    x = rng.standard_normal((batch, seq, heads, hd)).astype(np.float32)
    pos = np.array([0, 3, 17, 511, 2047], np.int32)
    ref = O.rope_neox(x, pos, batch, seq, heads, hd, 10000.0)
    out = torch.empty(x.size, dtype=torch.float32, device="cuda")
    ops.RoPE.apply_f32(dev(x), out, dev(pos), 10000.0, batch, seq, heads, hd)
    assert np.allclose(out.cpu().numpy().reshape(x.shape), ref.reshape(x.shape), rtol=5e-5, atol=5e-5)


@pytest.mark.parametrize("heads,kv_heads,hd,rows,past,window",
                         [(8, 2, 64, 5, 37, 0), (4, 4, 128, 1, 300, 0), (8, 1, 64, 3, 10, 0),
                          (4, 2, 128, 4, 60, 16), (2, 1, 32, 2, 5, 0), (2, 2, 256, 2, 70, 0)])
def test_attention_f32_vs_oracle(heads, kv_heads, hd, rows, past, window):
    rng = np.random.default_rng(heads * 100 + past)
    q = rng.standard_normal((rows, heads * hd)).astype(np.float32)
    k = rng.standard_normal((past + rows, kv_heads * hd)).astype(np.float32)
    v = rng.standard_normal((past + rows, kv_heads * hd)).astype(np.float32)
    ref = O.attention(q, k, v, rows, past, heads, kv_heads, hd, window)
    got = ops.attention(dev(q), dev(k), dev(v), past=past, heads=heads, kv_heads=kv_heads,
                        head_dim=hd, window=window).cpu().numpy()
    assert np.allclose(got, ref, rtol=2e-5, atol=2e-5)


# ---------------------------------------------------------------- prefill GEMM
@pytest.mark.parametrize("qt", [Q4_0, Q4_1, Q8_0])
@pytest.mark.parametrize("K,N,M", [(128, 128, 128), (256, 256, 200), (4096, 512, 512),
                                   (1024, 384, 1), (2048, 1280, 129),
                                   # GEMV fallback shapes (K % 64 or N % 128 != 0)
                                   (96, 64, 40), (160, 96, 70)])
def test_qgemm_vs_oracle(qt, K, N, M):
    raw = quant_matrix(qt, K, N, seed=K + N + M + qt)
    x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    y = ops.qgemm(dev(raw), qt, dev(x), N).cpu().numpy()
    check_gemv(y, ref_gemv(qt, LAYOUT_B, raw, K, N, x))


@pytest.mark.parametrize("qt", [Q4_0, Q8_0])
def test_qgemm_sweep_shape_512_rows(qt):
    """The sweep's GEMM case (M = 512) on the 7B FFN shape, against float64."""
    K, N, M = 4096, 14336, 512
    raw = quant_matrix(qt, K, N, seed=9)
    W = dev(O.dequantize(raw.tobytes(), qt, K * N).astype(np.float32).reshape(K, N))
    x = dev(np.random.default_rng(2).standard_normal((M, K)).astype(np.float32))
    y = ops.qgemm(dev(raw), qt, x, N)
    ref = (x.double() @ W.double()).cpu().numpy()
    check_gemv(y.cpu().numpy(), ref)


def test_qgemm_matches_gemv_rows():
    """The tensor-core GEMM and the 32-row GEMV agree on the same rows."""
    K, N, M = 2048, 1024, 96
    raw = quant_matrix(Q4_0, K, N, seed=4)
    x = dev(np.random.default_rng(8).standard_normal((M, K)).astype(np.float32))
    a = ops.qgemm(dev(raw), Q4_0, x, N)
    b = ops.qgemv(dev(raw), Q4_0, LAYOUT_B, x, N)
    scale = b.abs().max().item()
    assert (a - b).abs().max().item() <= 1e-5 * scale


# ---------------------------------------------------------------- K-quant dequant
def _k_blocks(qt, nb, seed):
    rng = np.random.default_rng(seed)
    S = 144 if qt == 12 else 210
    raw = rng.integers(0, 256, size=(nb, S), dtype=np.uint8)
    d = rng.choice(np.array([0.0123, -0.5, 3e-5, 1.0, 2.0], np.float16), (nb, 2))
    if qt == 12:
        raw[:, 12:16] = d.view(np.uint8).reshape(nb, 4)
    else:
        raw[:, 208:210] = d[:, :1].view(np.uint8).reshape(nb, 2)
    return raw.reshape(-1)


@pytest.mark.parametrize("qt", [12, 14])  # Q4_K, Q6_K
def test_k_quant_dequant_bit_exact(qt):
    nb = 4000
    raw = _k_blocks(qt, nb, qt)
    n = nb * 256 - 77
    ref = O.dequantize(raw.tobytes(), qt, n)
    got = ops.dequantize(dev(raw), qt, n).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_k_quant_short_buffer_and_stubs():
    with pytest.raises(WoollyError) as e:
        ops.dequantize(dev(np.zeros(143, np.uint8)), 12, 256)
    assert e.value.code == _lib.WL_ERR_INVALID_FORMAT
    for qt in (6, 7, 13, 15):  # Q5_0, Q5_1, Q5_K, Q8_K: zeros as the reference's stubs
        out = ops.dequantize(dev(np.full(400, 7, np.uint8)), qt, 256)
        assert not out.any().item()


def _tp_reduce(h, w, slots, counters, expect, err):
    rows, dim = h.shape
    T = slots.shape[0]
    y = torch.empty(2, rows, dim, dtype=torch.float16, device="cuda")
    _lib.check(_lib.lib().wl_tp_reduce_rmsnorm(
        h.data_ptr(), w.data_ptr(), rows, dim, 1e-5, slots.data_ptr(), T, counters.data_ptr(),
        expect, y.data_ptr(), rows * dim, err.data_ptr(), None))
    torch.cuda.synchronize()
    return y


@pytest.mark.parametrize("T,rows", [(1, 1), (2, 5), (3, 16), (8, 32)])
def test_tp_reduce_rmsnorm(T, rows):
    """The reduce side of the tensor-parallel exchange with T simulated ranks
    whose partial rows and arrival counts are written from the host: h gets
    the rank-ordered f32 sum (bit-exact), the output the RMSNorm of it
    (tensor_utils.rs:446-480), and the counters are re-armed to zero."""
    dim, expect = 4096, 37
    rng = np.random.default_rng(T * 100 + rows)
    h0 = rng.standard_normal((rows, dim)).astype(np.float32)
    parts = rng.standard_normal((T, 32, dim)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    h = dev(h0)
    slots = dev(parts)
    counters = torch.zeros(T + 1, dtype=torch.int32, device="cuda")
    counters[:T] = expect
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = _tp_reduce(h, dev(w), slots, counters, expect, err)
    ref_h = h0.copy()
    for r in range(T):
        ref_h = (ref_h + parts[r, :rows]).astype(np.float32)
    assert np.array_equal(h.cpu().numpy(), ref_h)
    rms = np.sqrt((ref_h.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-5)
    ref_y = ref_h / rms * w
    got = y[0].float() + y[1].float()
    assert np.abs(got.cpu().numpy() - ref_y).max() <= 1e-5 * np.abs(ref_y).max()
    assert int(err.item()) == 0
    assert counters.cpu().tolist() == [0] * (T + 1)


def test_tp_reduce_wait_gives_up():
    """Failure detection without a GPU fault: one simulated rank never
    finishes (its counter stays one short), the bounded wait gives up after
    about a second with bit 8 in the error word, and the context stays usable."""
    dim, T, rows, expect = 1024, 2, 2, 5
    h = torch.zeros(rows, dim, device="cuda")
    slots = torch.zeros(T, 32, dim, device="cuda")
    w = torch.ones(dim, device="cuda")
    counters = torch.zeros(T + 1, dtype=torch.int32, device="cuda")
    counters[0] = expect
    counters[1] = expect - 1
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    _tp_reduce(h, w, slots, counters, expect, err)
    assert int(err.item()) & 8
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum().item()) == 8.0
    # the counters re-arm to 0 (the short one does not wrap around), so the
    # next exchange waits for its own arrivals and reads the right slots
    assert counters.cpu().tolist() == [0] * (T + 1)
    rng = np.random.default_rng(3)
    parts = rng.standard_normal((T, 32, dim)).astype(np.float32)
    h0 = rng.standard_normal((rows, dim)).astype(np.float32)
    h.copy_(dev(h0))
    slots.copy_(dev(parts))
    counters[:T] = expect
    err.zero_()
    _tp_reduce(h, w, slots, counters, expect, err)
    assert int(err.item()) == 0
    ref_h = h0.copy()
    for r in range(T):
        ref_h = (ref_h + parts[r, :rows]).astype(np.float32)
    assert np.array_equal(h.cpu().numpy(), ref_h)
    assert counters.cpu().tolist() == [0] * (T + 1)



@pytest.mark.parametrize("qt", [Q4_0, Q4_1, Q8_0])
@pytest.mark.parametrize("K,N,M", [(256, 384, 70), (1024, 512, 300)])
def test_qgemm_tiled_vs_oracle(qt, K, N, M):
    """wl_qgemm_tiled: the tcgen05 GEMM streaming the tiled copy (bulk copies)
    against the restatement."""
    raw = quant_matrix(qt, K, N, seed=K + N + M + qt + 1)
    x = np.random.default_rng(M + 1).standard_normal((M, K)).astype(np.float32)
    tiled = ops.qtile(dev(raw), qt, K, N)
    y = ops.qgemm_tiled(tiled, qt, ops.split_planes(dev(x)), N).cpu().numpy()
    check_gemv(y, ref_gemv(qt, LAYOUT_B, raw, K, N, x))
