"""Model-level parity: the CUDA runtime vs the CPU oracle on seeded synthetic
GGUF models (GPU).

The bar (north_star): per-step teacher-forced logits within max-abs 1e-2 of
the oracle and top-1 agreement >= 99%.  Prompts are uniform random ids;
decode steps feed pre-drawn ids (teacher forcing), not the argmax.
"""
import os

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from woolly_b200 import Q4_0, WoollyError, _lib  # noqa: E402
from woolly_b200.gguf import write_synthetic  # noqa: E402
from woolly_b200.model import CudaTransformer, Session  # noqa: E402

LOGIT_TOL = 1e-2
TOP1_MIN = 0.99
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def compare(got, ref, what=""):
    got = np.asarray(got, np.float32).reshape(ref.shape)
    err = np.abs(got - ref).max()
    top1 = np.mean(got.reshape(-1, ref.shape[-1]).argmax(-1) == ref.reshape(-1, ref.shape[-1]).argmax(-1))
    assert err <= LOGIT_TOL, f"{what}: max-abs {err}"
    assert top1 >= TOP1_MIN, f"{what}: top-1 agreement {top1}"
    return err, top1


def teacher_forced(path, prompts, steps, seed=0, oracle_kw=None, **model_kw):
    """Prefill each prompt, then `steps` batched decode steps; returns the
    per-step logits of the GPU path and of the oracle."""
    rng = np.random.default_rng(seed + 1_000_000)
    m = CudaTransformer(path, **model_kw)
    V = m.vocab_size()
    forced = rng.integers(0, V, size=(steps, len(prompts)), dtype=np.uint32)
    sess = [Session(m) for _ in prompts]
    gpu_pref = m.forward_sessions(sess, prompts, all_logits=True)
    gpu_steps = []
    for t in range(steps):
        out = m.forward_sessions(sess, [[int(i)] for i in forced[t]])
        gpu_steps.append(np.stack(out))
    for s in sess:
        s.close()
    m.close()
    om = O.Model(path, **(oracle_kw or {}))
    kvs = [om.new_kv(max(len(p) for p in prompts) + steps + 1) for _ in prompts]
    or_pref = [om.forward(kv, p, all_rows=True) for kv, p in zip(kvs, prompts)]
    or_steps = [om.decode_batch(kvs, forced[t]) for t in range(steps)]
    om.close()
    return gpu_pref, np.stack(gpu_steps), or_pref, np.stack(or_steps)


def run_parity(path, prompts, steps, oracle_kw=None, **model_kw):
    gp, gs, op, os_ = teacher_forced(path, prompts, steps, oracle_kw=oracle_kw, **model_kw)
    for i, (a, b) in enumerate(zip(gp, op)):
        compare(a, b, f"prefill session {i}")
    compare(gs, os_, "decode steps")


def test_golden_tiny_forward(tmp_path):
    g = np.load(os.path.join(GOLD, "tiny_forward.npz"))
    import json
    spec = json.loads(str(g["spec"]))
    p = write_synthetic(str(tmp_path / "tiny.gguf"), **spec)
    m = CudaTransformer(p, max_sessions=2, max_context=64)
    logits = m.forward(g["ids"].tolist())
    m.close()
    compare(logits.reshape(g["logits"].shape), g["logits"], "golden tiny forward")


@pytest.mark.parametrize("name", ["gqa_q4_0", "mha_q4_1", "gqa_q8_0", "tied_q4_0"])
def test_teacher_forced_parity(tiny_models, name):
    prompts = [[1, 2, 3, 4, 5, 6, 7], [100, 200], list(range(40, 73))]
    run_parity(tiny_models[name], prompts, steps=12, max_sessions=4, max_context=128)


def test_wide_batch_decode_parity(tmp_path):
    """16 sessions x 16 KV heads = 256 (KV head, row) pairs per decode step,
    at least one per SM: the attention runs 1-page rounds with context splits
    and the combine kernel, the bs16 decode configuration of 7B-shape models."""
    p = write_synthetic(str(tmp_path / "wide.gguf"), hidden=1024, layers=2, heads=16,
                        kv_heads=16, ff=1024, vocab=512, weight_type=Q4_0, seed=11)
    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, 512, int(n)).tolist() for n in rng.integers(20, 90, 16)]
    run_parity(p, prompts, steps=6, max_sessions=16, max_context=128, max_batch=16)


def test_batch_engine_matches_one_at_a_time(tiny_models):
    """Continuous batching (woolly_b200.engine) on the GPU runtime: five greedy
    requests through three session slots give the same tokens as generating
    them one at a time, except where the top two logits are within 1e-3
    (batched and single-row GEMVs sum in different orders)."""
    from woolly_b200.engine import BatchEngine, GenerationConfig
    rng = np.random.default_rng(21)
    prompts = [rng.integers(3, 1024, int(n)).tolist() for n in (5, 17, 2, 33, 9)]
    cfg = GenerationConfig(max_tokens=8, eos_below=0)
    runs = []
    for mb in (3, 1):
        m = CudaTransformer(tiny_models["gqa_q4_0"], max_sessions=3, max_context=64, max_batch=3)
        eng = BatchEngine(m, max_batch=mb, keep_logits=True)
        ids = [eng.submit(p, cfg) for p in prompts]
        eng.run()
        runs.append([eng.finished[i] for i in ids])
        eng.close()
        m.close()
    for a, b in zip(*runs):
        assert len(a.tokens) == len(b.tokens) == 8
        for t, (ta, tb) in enumerate(zip(a.tokens, b.tokens)):
            assert np.abs(a.logits[t] - b.logits[t]).max() <= 1e-3
            if ta != tb:
                top2 = np.sort(b.logits[t])[-2:]
                assert top2[1] - top2[0] <= 1e-3
                break


def test_batch_engine_vs_oracle(tiny_models):
    """Continuous batching against the oracle: five greedy requests through
    three session slots (sessions released and reused mid-run); every logit
    row the engine sampled from matches the oracle's full-prefix forward over
    the request's prompt and its own generated tokens, and every pick is that
    row's argmax."""
    from woolly_b200.engine import BatchEngine, GenerationConfig
    path = tiny_models["gqa_q4_0"]
    rng = np.random.default_rng(22)
    prompts = [rng.integers(3, 1024, int(n)).tolist() for n in (5, 17, 2, 33, 9)]
    cfg = GenerationConfig(max_tokens=8, eos_below=0)
    m = CudaTransformer(path, max_sessions=3, max_context=64, max_batch=3)
    eng = BatchEngine(m, max_batch=3, keep_logits=True)
    ids = [eng.submit(p, cfg) for p in prompts]
    eng.run()
    done = [eng.finished[i] for i in ids]
    eng.close()
    m.close()
    om = O.Model(path)
    for p, r in zip(prompts, done):
        assert len(r.tokens) == 8
        seq = p + list(r.tokens[:-1])
        ref = om.forward(om.new_kv(len(seq) + 1), seq, all_rows=True)[len(p) - 1:]
        got = np.stack(r.logits)
        compare(got, ref, "engine rows")
        for t, tok in enumerate(r.tokens):
            assert tok == int(np.flatnonzero(got[t] == got[t].max())[-1])
    om.close()


def test_decode_without_graphs_matches(tiny_models):
    prompts = [[9, 8, 7], [1]]
    run_parity(tiny_models["gqa_q4_0"], prompts, steps=5, max_sessions=2, max_context=64,
               use_graphs=0)


def test_rope_neox_parity(tiny_models):
    prompts = [list(range(3, 20)), [5, 6]]
    run_parity(tiny_models["gqa_q4_0"], prompts, steps=6, oracle_kw=dict(rope=1),
               max_sessions=2, max_context=64, rope_mode=_lib.ROPE_NEOX)


def test_sliding_window_parity(tiny_models):
    # window 16 from metadata; contexts run past it
    prompts = [list(range(10, 40)), [3] * 5]
    run_parity(tiny_models["swa_q4_1"], prompts, steps=20, oracle_kw=dict(window=16),
               max_sessions=2, max_context=128)


def test_long_prefill_chunked_and_paged(tiny_models):
    # a prompt longer than max_prefill runs in chunks; contexts cross many pages
    rng = np.random.default_rng(4)
    prompts = [rng.integers(0, 1024, 150).tolist()]
    run_parity(tiny_models["gqa_q4_0"], prompts, steps=3, max_sessions=1, max_context=200,
               max_prefill=64)


@pytest.mark.parametrize("spec", [
    # 8 query heads per KV head (the 70B grouping), head_dim 128, window 100
    dict(hidden=1024, layers=1, heads=8, kv_heads=1, ff=512, vocab=512, weight_type=Q4_0,
         sliding_window=100, seed=31),
    # MHA, head_dim 64, no window
    dict(hidden=512, layers=1, heads=8, kv_heads=8, ff=512, vocab=512, weight_type=Q4_0, seed=32),
])
def test_prefill_attention_tensor_core_parity(tmp_path, spec):
    """Prompt chunks of >= 16 rows take the tensor-core prefill attention:
    chunks of 90, 90 and 21 rows (max_prefill 90) and a 17-row prompt, whose
    key ranges start mid-block, cross the window and end inside a 64-key
    block, against the oracle's full-prefix forward."""
    p = write_synthetic(str(tmp_path / "pf.gguf"), **spec)
    rng = np.random.default_rng(spec["seed"])
    prompts = [rng.integers(0, spec["vocab"], 201).tolist(), rng.integers(0, spec["vocab"], 17).tolist()]
    okw = dict(window=spec["sliding_window"]) if spec.get("sliding_window") else None
    run_parity(p, prompts, steps=4, oracle_kw=okw, max_sessions=2, max_context=256, max_prefill=90)


def test_device_step_matches_host_step(tiny_models):
    m = CudaTransformer(tiny_models["gqa_q4_0"], max_sessions=4, max_context=64)
    a = [Session(m) for _ in range(3)]
    b = [Session(m) for _ in range(1)]
    for s in a:
        s.infer([1, 2, 3])
    ids = np.array([4, 5, 6], np.uint32)
    host = np.stack(m.forward_sessions(a, [[int(i)] for i in ids]))
    for s in a:
        s.reset()
        s.infer([1, 2, 3])
    d_ids = torch.from_numpy(ids.view(np.int32)).cuda()
    d_log = torch.empty(3, m.vocab_size(), device="cuda")
    torch.cuda.synchronize()
    m.decode_step_device(a, d_ids.data_ptr(), d_log.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.abs(d_log.cpu().numpy() - host).max() <= 1e-5
    assert [len(s) for s in a] == [4, 4, 4]
    for s in a + b:
        s.close()
    m.close()


def test_errors(tiny_models):
    m = CudaTransformer(tiny_models["mha_q4_1"], max_sessions=2, max_context=16, max_batch=2)
    s = Session(m)
    with pytest.raises(WoollyError) as e:
        s.infer([512])  # vocab is 512
    assert e.value.code == _lib.WL_ERR_TOKEN_OUT_OF_RANGE
    with pytest.raises(WoollyError) as e:
        s.infer([])
    assert e.value.code == _lib.WL_ERR_INVALID_ARGUMENT
    s.infer(list(range(16)))
    with pytest.raises(WoollyError) as e:
        s.infer([1])
    assert e.value.code == _lib.WL_ERR_CONTEXT_FULL
    s2 = Session(m)
    with pytest.raises(WoollyError) as e:
        Session(m)
    assert e.value.code == _lib.WL_ERR_OUT_OF_MEMORY
    s.reset()
    assert len(s) == 0
    s.infer([1, 2])
    s.close()
    s2.close()
    m.close()
    with pytest.raises(WoollyError) as e:
        CudaTransformer("/nonexistent.gguf")
    assert e.value.code == _lib.WL_ERR_IO


def test_tinyllama_config_teacher_forced(tmp_path):
    """TinyLlama-1.1B shape, Q4_0, 128-token prompt + 128
    teacher-forced decode steps at batch 1, against the oracle."""
    p = write_synthetic(str(tmp_path / "tinyllama.gguf"), hidden=2048, layers=22, heads=32,
                        kv_heads=4, ff=5632, vocab=32000, weight_type=Q4_0, seed=1)
    prompt = np.random.default_rng(1 + 1_000_000).integers(0, 32000, 128).tolist()
    gp, gs, op, os_ = teacher_forced(p, [prompt], 128, seed=2, max_sessions=1, max_context=512,
                                     max_batch=1)
    e1, t1 = compare(gp[0], op[0], "tinyllama prefill")
    e2, t2 = compare(gs, os_, "tinyllama decode")
    print(f"tinyllama parity: prefill max-abs {e1:.2e} top1 {t1:.3f}; decode max-abs {e2:.2e} top1 {t2:.3f}")


@pytest.mark.parametrize("name", ["gqa_q4_0", "mha_q4_1", "gqa_q8_0", "tied_q4_0"])
@pytest.mark.parametrize("rope", [0, 1])
def test_ggml_layout_parity(tiny_models, name, rope):
    """The forward on weights in ggml orientation (llama.cpp checkpoints:
    every 2-D weight as ne1 rows of ne0, token_embd one row per token,
    quantized_matvec's layout, quantization.rs:1100-1163), with and without
    NeoX RoPE, against the oracle reading the same file the same way."""
    prompts = [[1, 2, 3, 4, 5, 6, 7], [100, 200], list(range(40, 73))]
    run_parity(tiny_models[name], prompts, steps=8, oracle_kw=dict(layout_a=1, rope=rope),
               max_sessions=4, max_context=128, ggml_layout=1,
               rope_mode=_lib.ROPE_NEOX if rope else _lib.ROPE_OFF)


def test_ggml_layout_tinyllama_rope(tmp_path):
    """TinyLlama shape in ggml orientation with RoPE on (how a llama.cpp
    checkpoint of it runs), 64 prompt tokens + 32 teacher-forced steps."""
    p = write_synthetic(str(tmp_path / "tinyllama.gguf"), hidden=2048, layers=22, heads=32,
                        kv_heads=4, ff=5632, vocab=32000, weight_type=Q4_0, seed=3)
    prompt = np.random.default_rng(3).integers(0, 32000, 64).tolist()
    gp, gs, op, os_ = teacher_forced(p, [prompt], 32, seed=4, oracle_kw=dict(layout_a=1, rope=1),
                                     max_sessions=1, max_context=128, max_batch=1, ggml_layout=1,
                                     rope_mode=_lib.ROPE_NEOX)
    e1, _ = compare(gp[0], op[0], "ggml tinyllama prefill")
    e2, _ = compare(gs, os_, "ggml tinyllama decode")
    print(f"ggml-orientation tinyllama (rope on): prefill max-abs {e1:.2e}, decode {e2:.2e}")


def test_inference_engine_api_on_the_runtime(tiny_models):
    """woolly-core's InferenceEngine / InferenceSession mirror over the CUDA
    runtime: a named session keeps its context across infer() calls, and its
    logits equal the Model-level forward of the whole sequence."""
    from woolly_b200.model import InferenceEngine
    m = CudaTransformer(tiny_models["gqa_q4_0"], max_sessions=3, max_context=64)
    eng = InferenceEngine()
    eng.load_model(m)
    s = eng.create_session()
    V = m.vocab_size()
    a = eng.infer([3, 4, 5], s.id()).reshape(-1, V)
    b = eng.infer([6, 7], s.id()).reshape(-1, V)
    full = m.forward([3, 4, 5, 6, 7]).reshape(-1, V)
    assert np.abs(np.concatenate([a, b]) - full).max() <= 1e-3
    assert s.token_history() == [3, 4, 5, 6, 7]
    s.deactivate()
    eng.cleanup_sessions()
    assert eng.list_sessions() == []
    m.close()
