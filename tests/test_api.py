"""woolly-core's engine / session API as mirrored in woolly_b200.model
(engine.rs:15-246, session.rs:118-330), driven with a fake device session so
that it runs on the CPU."""
import numpy as np
import pytest

from woolly_b200 import WoollyError, _lib
from woolly_b200.model import InferenceEngine

V = 8


class FakeModel:
    def name(self): return "fake"
    def model_type(self): return "llama"
    def vocab_size(self): return V
    def context_length(self): return 64
    def hidden_size(self): return 16
    def num_layers(self): return 2
    def num_heads(self): return 2


class FakeBackend:
    """Logits row t = position of token t in the session (so a session's
    history shows in its output)."""

    def __init__(self):
        self.n = 0
        self.closed = False

    def infer(self, tokens):
        rows = np.zeros((len(tokens), V), np.float32)
        for i in range(len(tokens)):
            rows[i, (self.n + i) % V] = 1.0
        self.n += len(tokens)
        return rows.reshape(-1)

    def reset(self):
        self.n = 0

    def close(self):
        self.closed = True


def make():
    eng = InferenceEngine(session_factory=FakeBackend)
    eng.load_model(FakeModel())
    return eng


def test_no_model_loaded():
    eng = InferenceEngine(session_factory=FakeBackend)
    with pytest.raises(WoollyError) as e:
        eng.infer([1, 2])
    assert "No model loaded" in str(e.value)
    assert eng.model_info() is None


def test_sessions_by_id_keep_their_context():
    eng = make()
    s = eng.create_session()
    a = eng.infer([5, 6, 7], s.id()).reshape(3, V)
    b = eng.infer([8], s.id()).reshape(1, V)
    assert a.argmax(1).tolist() == [0, 1, 2] and b.argmax(1).tolist() == [3]
    assert s.tokens_processed() == 4 and s.token_history() == [5, 6, 7, 8]
    # no id: a new registered session (engine.rs:90-105)
    c = eng.infer([1, 1]).reshape(2, V)
    assert c.argmax(1).tolist() == [0, 1]
    info = eng.list_sessions()
    assert len(info) == 2 and info[0]["id"] == s.id() and info[0]["tokens_processed"] == 4
    assert eng.model_info()["vocab_size"] == V


def test_errors_follow_the_reference():
    eng = make()
    with pytest.raises(WoollyError) as e:
        eng.infer([1], "no-such-session")
    assert e.value.code == _lib.WL_ERR_INVALID_ARGUMENT and "Session not found" in str(e.value)
    s = eng.create_session("fixed-id")
    assert s.id() == "fixed-id"
    with pytest.raises(WoollyError):
        s.infer([])
    s.deactivate()
    with pytest.raises(WoollyError) as e:
        s.infer([1])
    assert "not active" in str(e.value)


def test_clear_batch_and_cleanup():
    eng = make()
    s = eng.create_session()
    out = s.infer_batch([[1, 2], [3]])
    assert [o.reshape(-1, V).argmax(1).tolist() for o in out] == [[0, 1], [2]]
    s.clear()
    assert s.tokens_processed() == 0 and s.infer([9]).reshape(1, V).argmax(1).tolist() == [0]
    t = eng.create_session()
    t.deactivate()
    eng.cleanup_sessions()
    assert [i["id"] for i in eng.list_sessions()] == [s.id()]
    assert t._s.closed and not s._s.closed
