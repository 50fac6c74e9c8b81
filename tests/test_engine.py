"""Continuous-batching engine and the server's sampling rules (CPU).

The engine is exercised with a fake model whose logits for a session depend
only on that session's own token history, so batched generation must equal
one-request-at-a-time generation exactly; the sampler is checked against the
reference's rules (woolly-server/src/handlers/inference.rs:441-654).
"""
import numpy as np
import pytest

from woolly_b200 import _lib
from woolly_b200.engine import (BatchEngine, GenerationConfig, apply_top_k, apply_top_p,
                                sample_from_distribution, sample_next_token,
                                softmax_with_temperature)

V = 50


class FakeSession:
    def __init__(self, model):
        self.model = model
        self.hist = []
        model.open += 1

    def __len__(self):
        return len(self.hist)

    def close(self):
        self.model.open -= 1


class FakeModel:
    """Next-token logits peak at (7 * sum(history) + len(history)) % V."""

    def __init__(self, max_batch=4, max_sessions=4, max_context=64):
        self.max_batch, self.max_sessions, self.max_context = max_batch, max_sessions, max_context
        self.open = 0
        self.calls = []

    def vocab_size(self):
        return V

    def new_session(self):
        if self.open >= self.max_sessions:
            raise _lib.WoollyError(_lib.WL_ERR_OUT_OF_MEMORY, "no free session slot")
        return FakeSession(self)

    @staticmethod
    def row(hist):
        peak = (7 * sum(hist) + len(hist)) % V
        return -np.abs(np.arange(V, dtype=np.float32) - peak)

    def forward_sessions(self, sessions, ids):
        assert len(sessions) <= self.max_batch
        self.calls.append([len(i) for i in ids])
        out = []
        for s, t in zip(sessions, ids):
            assert len(s) + len(t) <= self.max_context
            s.hist += list(t)
            out.append(self.row(s.hist))
        return out


def sequential(prompt, cfg, max_context=64):
    hist, toks = list(prompt), []
    rng = np.random.default_rng(cfg.seed)
    while True:
        tok = sample_next_token(FakeModel.row(hist), cfg, rng)
        toks.append(tok)
        if len(toks) >= cfg.max_tokens or (cfg.eos_below and tok < cfg.eos_below):
            return toks
        if len(hist) + 1 > max_context:
            return toks
        hist.append(tok)


def make_engine(m, **kw):
    return BatchEngine(m, session_factory=m.new_session, **kw)


def test_batched_equals_sequential():
    m = FakeModel(max_batch=3, max_sessions=3)
    eng = make_engine(m)
    rng = np.random.default_rng(0)
    reqs = []
    for i in range(7):
        prompt = rng.integers(3, V, int(rng.integers(1, 9))).tolist()
        cfg = GenerationConfig(max_tokens=int(rng.integers(1, 12)), eos_below=0)
        reqs.append((eng.submit(prompt, cfg), prompt, cfg))
    out = eng.run()
    for rid, prompt, cfg in reqs:
        assert out[rid] == sequential(prompt, cfg)
    assert m.open == 0
    # decode steps really were batched, and never above max_batch
    assert max(len(c) for c in m.calls) == 3


def test_requests_join_between_steps():
    m = FakeModel(max_batch=4, max_sessions=4)
    eng = make_engine(m)
    cfg = GenerationConfig(max_tokens=6, eos_below=0)
    a = eng.submit([5, 6, 7], cfg)
    eng.step()
    eng.step()
    b = eng.submit([9], cfg)  # arrives while a is decoding
    out = eng.run()
    assert out[a] == sequential([5, 6, 7], cfg)
    assert out[b] == sequential([9], cfg)


def test_waits_for_session_slots():
    m = FakeModel(max_batch=8, max_sessions=2)
    eng = make_engine(m)
    cfg = GenerationConfig(max_tokens=3, eos_below=0)
    ids = [eng.submit([10 + i], cfg) for i in range(5)]
    out = eng.run()
    assert [out[i] for i in ids] == [sequential([10 + i], cfg) for i in range(5)]
    assert m.open == 0


def test_stop_rules():
    m = FakeModel(max_context=8)
    eng = make_engine(m)
    r_ctx = eng.submit([20, 21, 22, 23, 24], GenerationConfig(max_tokens=50, eos_below=0))
    r_long = eng.submit(list(range(3, 11)), GenerationConfig(max_tokens=5, eos_below=0))
    eng.run()
    f = eng.finished
    # 5 prompt tokens + fed-back tokens fill the 8-token context after 4 tokens
    assert f[r_ctx].reason == "context" and len(f[r_ctx].tokens) == 4
    assert f[r_long].reason == "context" and f[r_long].tokens == []  # prompt fills the context
    # EOS: after prompt [1]*25 the peak is (7*25 + 25) % 50 = 0 < 3
    m2 = FakeModel(max_context=64)
    eng2 = make_engine(m2)
    r_eos = eng2.submit([1] * 25, GenerationConfig(max_tokens=10))
    eng2.run()
    assert eng2.finished[r_eos].reason == "eos" and eng2.finished[r_eos].tokens == [0]
    with pytest.raises(ValueError):
        eng.submit([])


def test_softmax_with_temperature_floor():
    x = np.array([1.0, 2.0, 3.0], np.float32)
    p = softmax_with_temperature(x, 0.0)  # floored at 0.01
    e = np.exp((x - 3.0) / np.float32(0.01))
    assert np.allclose(p, e / e.sum())
    assert np.allclose(softmax_with_temperature(x, 1.0), np.exp(x - 3) / np.exp(x - 3).sum())


def test_top_k_and_top_p():
    p = np.array([0.1, 0.4, 0.2, 0.3], np.float32)
    k = apply_top_k(p, 2)
    assert np.allclose(k, [0, 0.4 / 0.7, 0, 0.3 / 0.7])
    assert apply_top_k(p, 0) is p and apply_top_k(p, 4) is p
    t = apply_top_p(p, 0.5)  # 0.4 (<= 0.5), 0.4 + 0.3 > 0.5: keep two
    assert np.allclose(t, [0, 0.4 / 0.7, 0, 0.3 / 0.7])
    # no prefix exceeds p (mass 0.9 < 0.95): the reference keeps nothing
    q = np.array([0.5, 0.4], np.float32)
    assert apply_top_p(q, 0.95).tolist() == [0.0, 0.0]


def test_greedy_and_sampling_rules():
    cfg = GenerationConfig(temperature=0.0)
    rng = np.random.default_rng(0)
    # equal maxima: Rust's max_by keeps the last one
    assert sample_next_token(np.array([1, 3, 3, 0], np.float32), cfg, rng) == 2
    # eight equal probabilities: top-p 0.999999 keeps all eight (only the full
    # sum 1.0 exceeds it) and greedy takes the last of the equal maxima
    cfg_p = GenerationConfig(temperature=0.0, top_p=0.999999)
    assert sample_next_token(np.zeros(8, np.float32), cfg_p, rng) == 7
    # sample_from_distribution: first running sum above the draw; last index on none
    probs = np.array([0.2, 0.3, 0.5], np.float32)
    r1, r2 = np.random.default_rng(5), np.random.default_rng(5)
    u = np.float32(r2.random(dtype=np.float32))
    want = int(np.flatnonzero(np.cumsum(probs, dtype=np.float32) > u)[0])
    assert sample_from_distribution(probs, r1) == want
    assert sample_from_distribution(np.zeros(4, np.float32), np.random.default_rng(1)) == 3


def test_seeded_sampling_is_reproducible():
    cfg = GenerationConfig(temperature=0.8, top_k=10, top_p=0.9, seed=3, max_tokens=8, eos_below=0)
    runs = []
    for _ in range(2):
        m = FakeModel()
        eng = make_engine(m)
        rid = eng.submit([4, 5], cfg)
        runs.append(eng.run()[rid])
    assert runs[0] == runs[1] == sequential([4, 5], cfg)


def test_streaming_callbacks_and_generator():
    """Tokens reach the per-request callback as they are produced (in order,
    the last one flagged done with its reason), and stream() yields a
    request's tokens while other requests share the batched steps."""
    m = FakeModel(max_batch=3, max_sessions=3)
    eng = make_engine(m)
    seen = {}
    cfgs = [GenerationConfig(max_tokens=n, eos_below=0) for n in (4, 6)]
    rids = [eng.submit([i + 1, 2 * i + 3], c, on_token=lambda rid, tok, done, why:
                       seen.setdefault(rid, []).append((tok, done, why))) for i, c in enumerate(cfgs)]
    streamed = list(eng.stream([9, 8, 7], GenerationConfig(max_tokens=5, eos_below=0)))
    eng.run()
    for rid, c, p in zip(rids, cfgs, ([1, 3], [2, 5])):
        toks = [t for t, _, _ in seen[rid]]
        assert toks == eng.finished[rid].tokens == sequential(p, c)
        assert [d for _, d, _ in seen[rid]] == [False] * (c.max_tokens - 1) + [True]
        assert seen[rid][-1][2] == "length"
    assert streamed == sequential([9, 8, 7], GenerationConfig(max_tokens=5, eos_below=0))
