"""Pins the CPU oracle to the reference's own known-answer tests (CPU only).

KAT sources (woolly, read as text):
  crates/woolly-tensor/src/quantization.rs:1294-1386  dequant KATs, block sizes
  crates/woolly-gguf/src/loader.rs:676-682            align_offset table
  crates/woolly-gguf/src/tensor_info.rs:281-305       Q4_0 64x64 data_size = 2304
  crates/woolly-core/src/tensor_utils.rs:608-620      2x2 matmul = [19, 22, 43, 50]
plus an independent cross-check against gguf-py's dequantizers (llama.cpp's
Python package, present in this image) and numpy's IEEE f16 widening.
"""
import json
import os
import struct
import tempfile

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def blk_q4_0(d, qs):
    return struct.pack("<e", d) + bytes(qs)


def blk_q4_1(d, m, qs):
    return struct.pack("<ee", d, m) + bytes(qs)


def blk_q8_0(d, qs):
    return struct.pack("<e", d) + np.asarray(qs, dtype=np.int8).tobytes()


def test_q4_0_kat():  # quantization.rs:1294-1307
    out = O.dequantize(blk_q4_0(2.0, [0] * 16), O.Q4_0, 32)
    assert np.all(out == -16.0)


def test_q4_1_kat():  # quantization.rs:1310-1326
    out = O.dequantize(blk_q4_1(1.0, 5.0, [0x01] * 16), O.Q4_1, 32)
    assert np.all(out[:16] == 6.0) and np.all(out[16:] == 5.0)


def test_q8_0_kat():  # quantization.rs:1329-1344
    qs = [0] * 32
    qs[0], qs[1] = 10, -5
    out = O.dequantize(blk_q8_0(0.5, qs), O.Q8_0, 32)
    assert out[0] == 5.0 and out[1] == -2.5 and np.all(out[2:] == 0)


def test_block_sizes():  # quantization.rs:1347-1356, dequantize.rs:221-244
    assert [O.lib().or_type_size(t) for t in (2, 3, 6, 7, 8)] == [18, 20, 22, 24, 34]
    assert [O.lib().or_block_size(t) for t in (0, 2, 12, 14)] == [1, 32, 256, 256]


def test_dispatcher_two_blocks():  # quantization.rs:1359-1386
    data = blk_q4_0(1.0, [0x11] * 16) + blk_q4_0(2.0, [0x22] * 16)
    out = O.dequantize(data, O.Q4_0, 64)
    assert np.all(out[:32] == -7.0) and np.all(out[32:] == -12.0)


def test_batch_equals_scalar():  # quantization.rs:1389-1407
    data = b"".join(blk_q4_0(float(i + 1), [0] * 16) for i in range(8))
    out = O.dequantize(data, O.Q4_0, 256)
    assert np.array_equal(out, np.repeat(-8.0 * np.arange(1, 9), 32).astype(np.float32))


def test_align_offset():  # loader.rs:676-682
    for a, b in [(0, 0), (1, 32), (31, 32), (32, 32), (33, 64)]:
        assert O.lib().or_align_offset(a, 32) == b


def test_matmul_2x2():  # tensor_utils.rs:608-620
    y = O.matmul_b([1, 2, 3, 4], [5, 6, 7, 8], 2, 2)
    assert y.ravel().tolist() == [19.0, 22.0, 43.0, 50.0]


def test_f16_widening_exhaustive():
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([O.half_to_float(int(x)) for x in h], dtype=np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_buffer_too_small():  # dequantize.rs:295-301, :250-256
    with pytest.raises(ValueError):
        O.dequantize(b"\x00" * 17, O.Q4_0, 32)
    with pytest.raises(ValueError):
        O.dequantize(b"\x00" * 7, O.F32, 2)


def test_partial_block_truncates():  # dequantize.rs:324: result.truncate(nelements)
    out = O.dequantize(blk_q8_0(1.0, list(range(32))), O.Q8_0, 20)
    assert out.tolist() == [float(i) for i in range(20)]


@pytest.mark.parametrize("qt", [O.Q4_0, O.Q4_1, O.Q8_0])
def test_dequant_matches_gguf_py(qt):
    gguf = pytest.importorskip("gguf")
    from gguf import quants
    rng = np.random.default_rng(qt)
    ts = {O.Q4_0: 18, O.Q4_1: 20, O.Q8_0: 34}[qt]
    nb = 4096
    raw = rng.integers(0, 256, size=(nb, ts), dtype=np.uint8)
    # finite, varied scales (including subnormals and negatives)
    scales = rng.choice(np.array([1e-6, 3e-5, 0.01, 0.5, -2.0, 100.0, 6e-8], np.float16), nb * 2)
    raw[:, 0:2] = scales[:nb].view(np.uint8).reshape(nb, 2)
    if qt == O.Q4_1:
        raw[:, 2:4] = scales[nb:].view(np.uint8).reshape(nb, 2)
    mine = O.dequantize(raw.tobytes(), qt, nb * 32)
    theirs = quants.dequantize(raw.reshape(-1), gguf.GGMLQuantizationType(qt)).astype(np.float32)
    assert np.array_equal(mine, theirs.ravel())


def test_quantized_matvec_scalar_semantics():
    # layout A: y[r] = sum over blocks of (q-8)*d*x, Q4_1 unsupported
    rng = np.random.default_rng(3)
    m, k = 8, 64
    raw = rng.integers(0, 256, size=(m * k // 32, 18), dtype=np.uint8)
    raw[:, 0:2] = np.full(m * k // 32, 0.25, np.float16).view(np.uint8).reshape(-1, 2)
    x = rng.standard_normal(k).astype(np.float32)
    y = O.quantized_matvec(O.Q4_0, raw, x, m, k)
    W = O.dequantize(raw.tobytes(), O.Q4_0, m * k).reshape(m, k).astype(np.float64)
    assert np.allclose(y, W @ x, rtol=1e-5, atol=1e-5)
    with pytest.raises(ValueError):
        O.quantized_matvec(O.Q4_1, np.zeros(20 * 2, np.uint8), x, 1, 64)


def test_swiglu_modes():
    g = np.linspace(-3, 3, 16, dtype=np.float32)
    u = np.ones(16, np.float32)
    exact = O.swiglu(g, u, 0)
    assert np.allclose(exact, g / (1 + np.exp(-g.astype(np.float64))), atol=1e-6)
    approx = O.swiglu(g, u, 1)  # AVX2: exp(-g) ~ 1 - g, over full 8-lanes
    assert np.allclose(approx, g * (1 / (1 + (1 - g))), atol=1e-6)


def test_kat_fixture_file():
    """The KAT fixture file (tests/golden/kats.json) replays through the oracle."""
    with open(os.path.join(GOLD, "kats.json")) as f:
        kats = json.load(f)
    for k in kats["dequant"]:
        out = O.dequantize(bytes.fromhex(k["hex"]), k["type"], k["n"])
        assert out.tolist() == k["expect"], k["source"]


# ---------------------------------------------------------------- K-quants
# The reference's own woolly_gguf::dequantize formulas for Q4_K and Q6_K
# (crates/woolly-gguf/src/dequantize.rs:404-462, :465-537), transcribed here a
# second time in plain Python float32 arithmetic, independently of oracle.c.
Q4_K, Q5_K, Q6_K, Q8_K = 12, 13, 14, 15
F32 = np.float32


def py_q4_k(block: bytes, n: int) -> list:
    sc = []
    for i in range(8):
        src = (i * 3) // 2
        if i % 2 == 0:
            sc.append(block[src] & 63)
        else:
            sc.append(((block[src] >> 6) | ((block[src + 1] & 15) << 2)) & 63)
    d = F32(np.frombuffer(block[12:14], np.float16)[0])
    dmin = F32(np.frombuffer(block[14:16], np.float16)[0])
    out = []
    for i in range(min(n, 256)):
        q = block[16 + i // 2] & 0x0F if i % 2 == 0 else (block[16 + i // 2] >> 4) & 0x0F
        out.append(d * F32(sc[i // 32]) * F32(q) + dmin)
    return out


def py_q6_k(block: bytes, n: int) -> list:
    ql, qh, scales = block[0:128], block[128:192], block[192:208]
    d = F32(np.frombuffer(block[208:210], np.float16)[0])
    out = []
    for i in range(min(n, 256)):
        ql_idx = 64 * (i // 128) + 32 * ((i % 128) // 64) + 16 * ((i % 64) // 32) + (i % 16)
        qh_idx = 32 * (i // 128) + 16 * ((i % 128) // 64) + 8 * ((i % 64) // 32) + (i % 32) // 4
        sh = 2 * ((i % 32) % 4)
        q1e = (qh[qh_idx] >> sh) & 3
        q2e = (qh[qh_idx] >> (sh + 2)) & 3 if sh < 6 else (qh[qh_idx + 1] & 3 if qh_idx + 1 < 64 else 0)
        q1 = (ql[ql_idx] & 0x0F) | (q1e << 4)
        q2 = (ql[ql_idx] >> 4) | (q2e << 4)
        q = q1 if i < 128 else q2
        out.append(d * F32(scales[i // 16]) * F32(q - 32) / F32(64.0))
    return out


def k_blocks(qt, nb, seed):
    rng = np.random.default_rng(seed)
    S = 144 if qt == Q4_K else 210
    raw = rng.integers(0, 256, size=(nb, S), dtype=np.uint8)
    d = rng.choice(np.array([0.0123, -0.5, 3e-5, 1.0, 2.0], np.float16), (nb, 2))
    if qt == Q4_K:
        raw[:, 12:16] = d.view(np.uint8).reshape(nb, 4)
    else:
        raw[:, 208:210] = d[:, :1].view(np.uint8).reshape(nb, 2)
    return raw


@pytest.mark.parametrize("qt,fn", [(Q4_K, py_q4_k), (Q6_K, py_q6_k)])
def test_k_quant_oracle_matches_transcription(qt, fn):
    raw = k_blocks(qt, 24, 7 + qt)
    n = 24 * 256 - 100  # the last super-block is partial (result.truncate)
    got = O.dequantize(raw.tobytes(), qt, n)
    ref = []
    for b in range(24):
        ref += fn(raw[b].tobytes(), n - 256 * b)
    assert np.array_equal(got.view(np.uint32), np.array(ref, np.float32).view(np.uint32))


def test_q4_k_hand_values():
    # scale 0 = 1 (byte 0 low six bits), d = 1, dmin = 0.5; qs[0] = 0x21 -> q = 1, 2
    blk = bytearray(144)
    blk[0] = 1
    blk[12:14] = np.float16(1.0).tobytes()
    blk[14:16] = np.float16(0.5).tobytes()
    blk[16] = 0x21
    out = O.dequantize(bytes(blk), Q4_K, 256)
    assert out[0] == 1.5 and out[1] == 2.5 and out[2] == 0.5
    assert out[32] == 0.5  # scale 1 is 0


def test_k_quant_short_buffer_and_zero_stubs():
    with pytest.raises(ValueError):
        O.dequantize(b"\x00" * 143, Q4_K, 256)
    with pytest.raises(ValueError):
        O.dequantize(b"\x00" * 209, Q6_K, 256)
    for qt in (6, 7, Q5_K, Q8_K):  # Q5_0, Q5_1, Q5_K, Q8_K: zeros (dequantize.rs:539-607)
        assert not O.dequantize(b"\x01" * 400, qt, 256).any()


def test_layout_a_reads_ggml_rows():
    """Oracle option layout_a (ggml orientation, llama.cpp files): an F32
    model whose 2-D weights hold ggml rows (N rows of K for dims [K, N];
    token_embd as one row per token) gives bit-identical logits to the same
    weights stored in the reference's reading ([K][N]) with layout_a off."""
    import gguf_builder as gb
    d, L, H, KVH, ff, V = 64, 2, 4, 2, 96, 40
    kvd = d // H * KVH
    rng = np.random.default_rng(3)
    meta = [("general.architecture", gb.STR, "llama"), ("llama.embedding_length", gb.U32, d),
            ("llama.block_count", gb.U32, L), ("llama.attention.head_count", gb.U32, H),
            ("llama.attention.head_count_kv", gb.U32, KVH), ("llama.feed_forward_length", gb.U32, ff),
            ("llama.vocab_size", gb.U32, V), ("llama.context_length", gb.U32, 64),
            ("llama.attention.layer_norm_epsilon", gb.F32, 1e-5)]
    mats = [("token_embd.weight", d, V), ("output.weight", d, V)]
    vecs = [("output_norm.weight", d)]
    for l in range(L):
        vecs += [(f"blk.{l}.attn_norm.weight", d), (f"blk.{l}.ffn_norm.weight", d)]
        mats += [(f"blk.{l}.attn_q.weight", d, d), (f"blk.{l}.attn_k.weight", d, kvd),
                 (f"blk.{l}.attn_v.weight", d, kvd), (f"blk.{l}.attn_output.weight", d, d),
                 (f"blk.{l}.ffn_gate.weight", d, ff), (f"blk.{l}.ffn_up.weight", d, ff),
                 (f"blk.{l}.ffn_down.weight", ff, d)]
    tb, ta = [], []
    for name, n in vecs:
        v = (1 + 0.02 * rng.standard_normal(n)).astype(np.float32).tobytes()
        tb.append((name, [n], 0, len(v), v))
        ta.append((name, [n], 0, len(v), v))
    for name, K, N in mats:
        w = (0.1 * rng.standard_normal((K, N))).astype(np.float32)  # reference reading [K][N]
        tb.append((name, [K, N], 0, w.nbytes, w.tobytes()))
        ta.append((name, [K, N], 0, w.nbytes, np.ascontiguousarray(w.T).tobytes()))  # ggml rows
    paths = []
    for tag, ts in (("b", tb), ("a", ta)):
        p = os.path.join(tempfile.mkdtemp(), f"m_{tag}.gguf")
        with open(p, "wb") as f:
            f.write(gb.build(meta, ts))
        paths.append(p)
    ids = [3, 17, 5, 39, 0, 11]
    out = []
    for p, la in ((paths[0], 0), (paths[1], 1), (paths[1], 0)):
        m = O.Model(p, layout_a=la)
        out.append(m.forward(m.new_kv(16), ids, all_rows=True))
        m.close()
    assert np.array_equal(out[0], out[1])
    assert not np.allclose(out[0], out[2])  # the same bytes read the other way differ


@pytest.mark.parametrize("kw", [
    dict(hidden=256, layers=2, heads=4, kv_heads=2, ff=512, vocab=512, weight_type=O.Q4_0, seed=3),
    dict(hidden=256, layers=1, heads=2, kv_heads=2, ff=256, vocab=320, weight_type=O.Q4_1,
         sliding_window=16, seed=4),
    dict(hidden=512, layers=1, heads=4, kv_heads=1, ff=768, vocab=256, weight_type=O.Q8_0,
         tied=True, norm_eps=1e-6, rope_theta=5e5, seed=5),
    dict(hidden=128, layers=1, heads=2, kv_heads=1, ff=256, vocab=64, weight_type=O.F32,
         output_type=O.Q4_0, context_length=64, seed=6),
    # > 65536 values per tensor: several seed chunks
    dict(hidden=512, layers=1, heads=8, kv_heads=8, ff=1024, vocab=1024, weight_type=O.Q4_0, seed=9),
    # K-quants: Q4_K with Q6_K attn_v / ffn_down / output (the usual mix), and all-Q6_K
    dict(hidden=512, layers=1, heads=4, kv_heads=2, ff=768, vocab=1024, weight_type=O.Q4_K,
         vd_type=O.Q6_K, output_type=O.Q6_K, seed=10),
    dict(hidden=256, layers=1, heads=2, kv_heads=2, ff=512, vocab=512, weight_type=O.Q6_K, seed=11),
    # quantized token embeddings
    dict(hidden=256, layers=1, heads=2, kv_heads=2, ff=512, vocab=512, weight_type=O.Q4_0,
         embd_type=O.Q8_0, seed=12),
    dict(hidden=256, layers=1, heads=2, kv_heads=2, ff=512, vocab=512, weight_type=O.Q4_K,
         vd_type=O.Q6_K, embd_type=O.Q4_K, output_type=O.Q6_K, seed=13),
])
def test_oracle_writer_matches_product_writer(tmp_path, kw):
    """The oracle's own GGUF writer (used where the product library must not
    load) writes exactly the bytes of the product's wl_synth_gguf."""
    from woolly_b200.gguf import write_synthetic
    a = O.synth_gguf(str(tmp_path / "oracle.gguf"), **kw)
    b = write_synthetic(str(tmp_path / "product.gguf"), **kw)
    with open(a, "rb") as fa, open(b, "rb") as fb:
        assert fa.read() == fb.read()


@pytest.mark.parametrize("ty", [O.Q4_K, O.Q6_K])
def test_kquant_writer_blocks_read_back(ty):
    """The K-quant encoders target woolly's reading of the blocks
    (dequantize.rs:381-537): Q4_K reads back within one quantization step of
    the source values; Q6_K, whose reference reading takes values i and
    i + 16 of a 32-run from the same low nibble, still reads back values of
    the source's scale (same sign pattern for most of them)."""
    from woolly_b200.gguf import quantize, synth_normal
    x = synth_normal(7, 3, 256 * 64, 0.0, 0.02)
    q = quantize(ty, x)
    assert q.size == x.size // 256 * (144 if ty == O.Q4_K else 210)
    y = O.dequantize(q, ty, x.size)
    assert np.all(np.isfinite(y))
    if ty == O.Q4_K:
        step = (x.reshape(-1, 256).max(1) - x.reshape(-1, 256).min(1)) / 15
        assert np.all(np.abs(y - x).reshape(-1, 256).max(1) <= step * 1.01 + 1e-6)
    else:
        assert 0.5 < y.std() / x.std() < 2.0
        assert np.mean(np.sign(y) == np.sign(x)) > 0.7
