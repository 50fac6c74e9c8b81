"""GGUF parsing and the synthetic writer (CPU only).

Mirrors woolly-gguf's integration tests (crates/woolly-gguf/tests/
load_model.rs:148-360) against the product parser, and cross-checks both
parsers (product C++, oracle C) plus gguf-py's reader on written files.
"""
import struct

import numpy as np
import pytest

import gguf_builder as GB
import oracle as O
from woolly_b200 import Q4_0, Q4_1, Q8_0, WoollyError, _lib
from woolly_b200.gguf import GGMLType, GGUFLoader, quantize, write_synthetic


def test_load_empty_gguf():  # load_model.rs:148-169
    g = GGUFLoader.from_bytes(GB.build())
    h = g.header()
    assert (h.version, h.tensor_count, h.metadata_kv_count) == (3, 0, 0)
    assert g.tensors() == []


def test_load_with_metadata():  # load_model.rs:171-210
    md = [("general.architecture", GB.STR, "test_arch"), ("general.name", GB.STR, "Test Model"),
          ("general.quantization_version", GB.U32, 2), ("general.alignment", GB.U32, 32),
          ("test.bool_value", GB.BOOL, True), ("test.float_value", GB.F32, 3.14),
          ("test.array_value", GB.ARR, (GB.U32, [1, 2, 3]))]
    g = GGUFLoader.from_bytes(GB.build(md))
    assert g.header().metadata_kv_count == 7
    assert g.architecture() == "test_arch"
    assert g.get_str("general.name") == "Test Model"
    assert g.get_u32("general.quantization_version") == 2
    assert g.alignment() == 32
    assert abs(g.get_f32("test.float_value") - 3.14) < 1e-3
    assert g.get_u32("test.float_value") is None  # typed getters need the exact type


def test_load_with_tensors():  # load_model.rs:212-251
    t1 = bytes(range(16))
    t2 = bytes(range(32))
    data = GB.build([("general.architecture", GB.STR, "test")],
                    [("weight1", (4, 4), 0, 64, t1 + bytes(48)),
                     ("weight2", (4, 4, 2), 0, 128, t2 + bytes(96))])
    g = GGUFLoader.from_bytes(data)
    assert set(g.tensor_names()) == {"weight1", "weight2"}
    i1 = g.tensor_info("weight1")
    assert i1.shape == (4, 4) and i1.ggml_type == 0 and i1.n_elements == 16 and i1.data_size == 64
    assert g.tensor_info("weight2").n_elements == 32


def test_memory_mapped_tensor_access():  # load_model.rs:253-285
    vals = np.arange(16, dtype=np.float32)
    g = GGUFLoader.from_bytes(GB.build([("general.architecture", GB.STR, "test")],
                                       [("test_tensor", (4, 4), 0, 64, vals.tobytes())]))
    raw = g.tensor_data("test_tensor")
    assert raw.size == 64
    assert np.array_equal(raw.view(np.float32), vals)


def test_quantized_tensor_handling():  # load_model.rs:287-315
    g = GGUFLoader.from_bytes(GB.build([("general.architecture", GB.STR, "test")],
                                       [("quantized_weight", (64,), 2, 36, bytes(36))]))
    ti = g.tensor_info("quantized_weight")
    assert ti.ggml_type == GGMLType.Q4_0 and GGMLType(ti.ggml_type).is_quantized()
    assert ti.data_size == 36
    assert g.tensor_data("quantized_weight").size == 36


def test_error_handling(tmp_path):  # load_model.rs:317-345
    with pytest.raises(WoollyError) as e:
        GGUFLoader.from_path("/non/existent/file.gguf")
    assert e.value.code == _lib.WL_ERR_IO
    with pytest.raises(WoollyError) as e:
        GGUFLoader.from_bytes(b"BAD!" + bytes(20))
    assert e.value.code == _lib.WL_ERR_INVALID_MAGIC
    with pytest.raises(WoollyError) as e:
        GGUFLoader.from_bytes(b"GGUF" + struct.pack("<I", 999) + bytes(16))
    assert e.value.code == _lib.WL_ERR_UNSUPPORTED_VERSION
    # the oracle parser reports the same kinds
    assert O.gguf_status(b"BAD!" + bytes(20)) == 2
    assert O.gguf_status(b"GGUF" + struct.pack("<I", 999) + bytes(16)) == 3


def test_tensor_not_found():  # load_model.rs:347-360
    g = GGUFLoader.from_bytes(GB.build([("general.architecture", GB.STR, "test")]))
    with pytest.raises(WoollyError) as e:
        g.tensor_info("nope")
    assert e.value.code == _lib.WL_ERR_TENSOR_NOT_FOUND


def test_truncated_and_bad_type():
    full = GB.build([("general.architecture", GB.STR, "test")],
                    [("w", (32,), 2, 18, bytes(18))])
    for cut in (10, 30, 60):
        with pytest.raises(WoollyError) as e:
            GGUFLoader.from_bytes(full[:cut])
        assert e.value.code == _lib.WL_ERR_IO
    bad = GB.build([], [("w", (32,), 5, 18, bytes(18))])  # type 5 does not exist
    with pytest.raises(WoollyError) as e:
        GGUFLoader.from_bytes(bad)
    assert e.value.code == _lib.WL_ERR_INVALID_TENSOR_TYPE


def test_data_size_table():  # tensor_info.rs:281-305 (Q4_0 64x64 -> 2304 bytes)
    g = GGUFLoader.from_bytes(GB.build([], [("w", (64, 64), 2, 2304, bytes(2304))]))
    assert g.tensor_info("w").data_size == 2304


def test_model_config_defaults():  # model/loader.rs:104-156
    g = GGUFLoader.from_bytes(GB.build([("general.architecture", GB.STR, "llama"),
                                        ("llama.embedding_length", GB.U32, 64),
                                        ("llama.attention.head_count", GB.U32, 4)]))
    c = g.model_config()
    assert c["hidden_size"] == 64 and c["num_heads"] == 4
    assert c["vocab_size"] == 32000 and c["num_layers"] == 32 and c["context_length"] == 2048
    assert c["intermediate_size"] == 256 and c["layer_norm_epsilon"] == pytest.approx(1e-5)
    with pytest.raises(WoollyError):
        GGUFLoader.from_bytes(GB.build()).model_config()  # no architecture


def test_synthetic_writer_roundtrip(tmp_path):
    p = write_synthetic(str(tmp_path / "m.gguf"), hidden=256, layers=2, heads=4, kv_heads=2,
                        ff=512, vocab=512, weight_type=Q4_0, seed=7)
    g = GGUFLoader.from_path(p)
    c = g.model_config()
    assert (c["hidden_size"], c["num_layers"], c["num_heads"], c["vocab_size"],
            c["intermediate_size"]) == (256, 2, 4, 512, 512)
    assert g.tensor_info("blk.0.attn_k.weight").shape == (256, 128)
    assert g.tensor_info("token_embd.weight").shape == (256, 512)
    assert all(t.offset % 32 == 0 for t in g.tensors())
    # deterministic
    p2 = write_synthetic(str(tmp_path / "m2.gguf"), hidden=256, layers=2, heads=4, kv_heads=2,
                         ff=512, vocab=512, weight_type=Q4_0, seed=7)
    assert open(p, "rb").read() == open(p2, "rb").read()
    # gguf-py reads the same tensors and bytes
    gguf = pytest.importorskip("gguf")
    r = gguf.GGUFReader(p)
    names = {t.name: t for t in r.tensors}
    assert set(names) == set(g.tensor_names())
    t = names["blk.1.ffn_down.weight"]
    assert np.array_equal(np.asarray(t.data).view(np.uint8).ravel(),
                          g.tensor_data("blk.1.ffn_down.weight"))


@pytest.mark.parametrize("qt", [Q4_0, Q4_1, Q8_0])
def test_quantizer_error_bound(qt):
    rng = np.random.default_rng(qt)
    x = rng.standard_normal(32 * 256).astype(np.float32) * 0.02
    blocks = quantize(qt, x)
    y = O.dequantize(blocks.tobytes(), qt, x.size)
    xb = x.reshape(-1, 32)
    err = np.abs(y.reshape(-1, 32) - xb).max(axis=1)
    amax = np.abs(xb).max(axis=1)
    rng_b = xb.max(axis=1) - xb.min(axis=1)
    # Q4_0 clamps the far end (+8 -> 15), so its worst case is one full step
    bound = {Q4_0: amax / 8 * 1.0 + 1e-7, Q4_1: rng_b / 15 * 0.51 + 1e-6,
             Q8_0: amax / 127 * 0.51 + 1e-7}[qt] * 1.01
    assert np.all(err <= bound + 2e-3 * amax)
