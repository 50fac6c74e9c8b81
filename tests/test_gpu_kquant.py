"""K-quant (Q4_K / Q6_K) GEMV and model forward against the CPU oracle (GPU).

The values of a K-quant matrix are woolly_gguf::dequantize's reading of the
super-block bytes (dequantize.rs:381-537), which the oracle restates; the GPU
path computes from its tiled copy (codes plus the sub-block scale d*sc as an
exact f16 pair).  Same bars as the other types: GEMV within 4e-3 of max|ref|,
model logits within max-abs 1e-2 and top-1 >= 99%.
"""
import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from woolly_b200 import LAYOUT_A, LAYOUT_B, WoollyError, _lib  # noqa: E402
from woolly_b200 import ops  # noqa: E402
from woolly_b200.gguf import quantize, write_synthetic  # noqa: E402

Q4_K, Q6_K = 12, 14
SB = {Q4_K: 144, Q6_K: 210}
TILE_UNIT = {Q4_K: 22, Q6_K: 40}
GEMV_TOL = 4e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def random_superblocks(qt, nb, seed, scales=(1.3e-4, -2e-3, 6e-8, 0.5, 3e-5, 1.0)):
    """Any code and six-bit / eight-bit scale bytes, with d (and dmin) drawn
    from f16 values of very different magnitude (subnormal included)."""
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(nb, SB[qt]), dtype=np.uint8)
    d = rng.choice(np.array(scales, np.float16), nb).view(np.uint8).reshape(nb, 2)
    if qt == Q4_K:
        raw[:, 12:14] = d
        raw[:, 14:16] = rng.choice(np.array(scales, np.float16), nb).view(np.uint8).reshape(nb, 2)
    else:
        raw[:, 208:210] = d
    return raw.reshape(-1)


def ref_gemv(qt, raw, K, N, x):
    W = O.dequantize(raw.tobytes(), qt, K * N).astype(np.float64).reshape(K, N)
    return x.astype(np.float64) @ W


def check(y, ref):
    y = np.asarray(y, np.float64)
    scale = np.abs(ref).max()
    err = np.abs(y - ref).max()
    assert err <= GEMV_TOL * scale + 1e-6, (err, scale)


@pytest.mark.parametrize("qt", [Q4_K, Q6_K])
@pytest.mark.parametrize("K,N", [(512, 1024), (80, 256), (4096, 4096), (11008, 4096), (4096, 11008)])
@pytest.mark.parametrize("B", [1, 3, 5, 16, 33])
def test_kquant_qgemv_vs_oracle(qt, K, N, B):
    """Encoded N(0, 0.02) weights; a partial last stage (K = 80); LOC (B <= 4),
    one to three batch tiles and a second 32-row chunk (B = 33)."""
    rng = np.random.default_rng(K * 3 + N + qt)
    raw = quantize(qt, (rng.standard_normal(K * N) * 0.02).astype(np.float32))
    x = np.random.default_rng(B).standard_normal((B, K)).astype(np.float32)
    y = ops.qgemv(dev(raw), qt, LAYOUT_B, dev(x), N)
    check(y.cpu().numpy(), ref_gemv(qt, raw, K, N, x))


@pytest.mark.parametrize("qt", [Q4_K, Q6_K])
@pytest.mark.parametrize("B", [1, 16])
def test_kquant_any_bytes(qt, B):
    """Random super-block bytes: every scale field and code pattern, including
    the Q6_K bits that the reference reads twice."""
    K, N = 256, 2048
    raw = random_superblocks(qt, K * N // 256, seed=qt * 10 + B)
    x = np.random.default_rng(B + 3).standard_normal((B, K)).astype(np.float32)
    y = ops.qgemv(dev(raw), qt, LAYOUT_B, dev(x), N).cpu().numpy()
    check(y, ref_gemv(qt, raw, K, N, x))


@pytest.mark.parametrize("qt", [Q4_K, Q6_K])
def test_kquant_tiled_copy(qt):
    """wl_qtile_repack + wl_qgemv_tiled (the runtime's path) give wl_qgemv's
    result; the copy has the documented size."""
    K, N, B = 1024, 768, 12
    rng = np.random.default_rng(qt)
    raw = quantize(qt, (rng.standard_normal(K * N) * 0.02).astype(np.float32))
    x = dev(np.random.default_rng(1).standard_normal((B, K)).astype(np.float32))
    t = ops.qtile(dev(raw), qt, K, N)
    assert t.numel() == (N // 256) * ((K + 63) // 64) * 512 * TILE_UNIT[qt]
    y = ops.qgemv_tiled(t, qt, ops.split_planes(x), N)
    y0 = ops.qgemv(dev(raw), qt, LAYOUT_B, x, N)
    assert torch.equal(y, y0)


def test_kquant_rejects_bad_shapes():
    raw = dev(np.zeros(64 * 144, np.uint8))
    x = dev(np.zeros((1, 64), np.float32))
    with pytest.raises(WoollyError):
        ops.qgemv(raw, Q4_K, LAYOUT_B, x, 128)  # N % 256 != 0
    with pytest.raises(WoollyError):
        ops.qgemv(raw, Q4_K, LAYOUT_A, x, 256)  # layout A has no K-quant path
    assert _lib.lib().wl_qtile_bytes(Q6_K, 64, 288) == 0


@pytest.mark.parametrize("qt", [Q4_K, Q6_K])
@pytest.mark.parametrize("K,N,M", [(512, 1024, 64), (4096, 4096, 512), (4096, 11008, 200),
                                   (11008, 4096, 130), (80, 512, 96)])
def test_kquant_qgemm_vs_oracle(qt, K, N, M):
    """Prompts: the tcgen05 GEMM on the K-quant tiled copy (K % 64 == 0;
    partial row tiles M = 200, 130), and the 32-row GEMV chunks otherwise
    (K = 80)."""
    rng = np.random.default_rng(K + N + M + qt)
    raw = quantize(qt, (rng.standard_normal(K * N) * 0.02).astype(np.float32))
    x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float32)
    y = ops.qgemm(dev(raw), qt, dev(x), N).cpu().numpy()
    check(y, ref_gemv(qt, raw, K, N, x))
    if K % 64 == 0:
        t = ops.qtile(dev(raw), qt, K, N)
        y2 = ops.qgemm_tiled(t, qt, ops.split_planes(dev(x)), N).cpu().numpy()
        assert np.array_equal(y, y2)


def _parity(path, prompts, steps, **kw):
    from test_gpu_model import run_parity
    run_parity(path, prompts, steps, **kw)


@pytest.mark.parametrize("spec", [
    # the usual mix: Q4_K projections with Q6_K attn_v / ffn_down / output
    dict(hidden=512, layers=2, heads=4, kv_heads=2, ff=768, vocab=1024, weight_type=Q4_K,
         vd_type=Q6_K, output_type=Q6_K, seed=21),
    dict(hidden=512, layers=2, heads=4, kv_heads=4, ff=1024, vocab=768, weight_type=Q6_K, seed=22),
    dict(hidden=256, layers=2, heads=2, kv_heads=2, ff=512, vocab=512, weight_type=Q4_K, seed=23),
])
def test_kquant_model_teacher_forced_parity(tmp_path, spec):
    """Prefill (70- and 96-row prompts take the tensor-core GEMM, shorter ones
    32-row GEMV chunks) and batched decode on K-quant weights, fused q/k/v of
    mixed types included."""
    p = write_synthetic(str(tmp_path / "kq.gguf"), **spec)
    rng = np.random.default_rng(spec["seed"])
    prompts = [rng.integers(0, spec["vocab"], n).tolist() for n in (70, 9, 33, 96)]
    # 25 steps x 4 sessions: 100 decode rows, so that one top-1 flip on a
    # near tie (spec 3 has a decode row whose top-2 logits differ by 2e-6 in
    # the oracle itself) stays within the 99% bar
    _parity(p, prompts, steps=25, max_sessions=4, max_context=128, max_batch=4)


def test_kquant_device_decode_matches_host_step(tmp_path):
    """The graph-captured device decode step on a K-quant mix equals the host
    step (the mixed q/k/v launches are inside the captured sequence)."""
    from woolly_b200.model import CudaTransformer, Session
    p = write_synthetic(str(tmp_path / "kqd.gguf"), hidden=512, layers=2, heads=4, kv_heads=2,
                        ff=768, vocab=1024, weight_type=Q4_K, vd_type=Q6_K, output_type=Q6_K, seed=5)
    m = CudaTransformer(p, max_sessions=4, max_context=64, max_batch=4)
    a = [Session(m) for _ in range(2)]
    b = [Session(m) for _ in range(2)]
    for sa, sb, pr in zip(a, b, ([1, 2, 3], [7, 8, 9, 10])):
        sa.infer(pr)
        sb.infer(pr)
    ids = [11, 12]
    for _ in range(3):
        host = np.stack(m.forward_sessions(a, [[i] for i in ids]))
        dev_ids = m.decode_sample(b, ids)
        want = [int(np.flatnonzero(r == r.max())[-1]) for r in host]
        assert list(dev_ids) == want
        ids = want
    for s in a + b:
        s.close()
    m.close()


@pytest.mark.parametrize("spec", [
    # the Q4_K_M-style mix with a quantized embedding, as llama.cpp files hold it
    dict(hidden=512, layers=2, heads=4, kv_heads=2, ff=768, vocab=1024, weight_type=Q4_K,
         vd_type=Q6_K, output_type=Q6_K, embd_type=Q4_K, seed=41),
    dict(hidden=512, layers=1, heads=8, kv_heads=8, ff=512, vocab=512, weight_type=Q6_K,
         embd_type=Q6_K, seed=42),
])
@pytest.mark.parametrize("rope", [0, 1])
def test_kquant_ggml_orientation_parity(tmp_path, spec, rope):
    """K-quant weights and embedding in ggml orientation (rows of K values with
    256-value super-blocks along K; token_embd one row per token), with and
    without NeoX RoPE, against the oracle reading the file the same way."""
    p = write_synthetic(str(tmp_path / "kqa.gguf"), **spec)
    rng = np.random.default_rng(spec["seed"] + rope)
    prompts = [rng.integers(0, spec["vocab"], n).tolist() for n in (7, 40, 2)]
    _parity(p, prompts, steps=34, oracle_kw=dict(layout_a=1, rope=rope), max_sessions=3,
            max_context=128, ggml_layout=1,
            rope_mode=_lib.ROPE_NEOX if rope else _lib.ROPE_OFF)


@pytest.mark.parametrize("embd", [8, 12, 14])
def test_quantized_embedding_parity(tmp_path, embd):
    """token_embd.weight of a quantized type is dequantized on the device as
    woolly_gguf::dequantize reads it (bit-exact kernels) and the forward
    matches the oracle (woolly's orientation)."""
    p = write_synthetic(str(tmp_path / "qe.gguf"), hidden=512, layers=1, heads=4, kv_heads=2, ff=512,
                        vocab=512, weight_type=2, embd_type=embd, seed=43)
    rng = np.random.default_rng(embd)
    prompts = [rng.integers(0, 512, n).tolist() for n in (20, 5)]
    _parity(p, prompts, steps=50, max_sessions=2, max_context=96)
