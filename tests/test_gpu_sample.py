"""GPU next-token sampling (wl_sample) against the server's rules as
restated on the host in woolly_b200/engine.py (inference.rs:441-654).

The uniform draw of each row is given to both sides.  Greedy picks must be
identical.  Sampled picks must be identical except where the draw lies within
1e-5 of a cumulative boundary (the device sums in a fixed tree order, the
reference sequentially, so they can round a boundary differently)."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from woolly_b200 import ops  # noqa: E402
from woolly_b200.engine import GenerationConfig, apply_top_k, apply_top_p, \
    softmax_with_temperature  # noqa: E402


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def host_probs(logits, cfg):
    p = softmax_with_temperature(logits, cfg.temperature)
    if cfg.top_k > 0:
        p = apply_top_k(p, cfg.top_k)
    if cfg.top_p < 1.0:
        p = apply_top_p(p, cfg.top_p)
    return p


def host_pick(p, cfg, u):
    if cfg.temperature == 0.0:
        return int(np.flatnonzero(p == p.max())[-1])
    cum = np.cumsum(p, dtype=np.float32)
    hit = np.flatnonzero(cum > np.float32(u))
    return int(hit[0]) if hit.size else p.size - 1, cum


CASES = [
    dict(temperature=0.0),
    dict(temperature=0.7),
    dict(temperature=1.0, top_k=40),
    dict(temperature=0.8, top_p=0.9),
    dict(temperature=1.3, top_k=50, top_p=0.95),
    dict(temperature=0.0, top_k=5),
    dict(temperature=0.5, top_k=1),
    dict(temperature=1.0, top_p=0.3),
]


@pytest.mark.parametrize("V", [32000, 1000, 50])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_sample_matches_server_rules(V, case):
    kw = CASES[case]
    cfg = GenerationConfig(temperature=kw.get("temperature", 1.0), top_k=kw.get("top_k", 0),
                           top_p=kw.get("top_p", 1.0))
    rng = np.random.default_rng(V + 17 * case)
    rows = 24
    logits = (rng.standard_normal((rows, V)) * 3).astype(np.float32)
    logits[0, : V // 2] = logits[0, V // 2:]  # every value twice: ties for greedy/top-k/top-p
    logits[1, 3] = logits[1, 7] = logits[1].max() + 1.0  # a tied maximum
    u = rng.random(rows, dtype=np.float32)
    got = ops.sample(torch.from_numpy(logits).cuda(), cfg.temperature, cfg.top_k, cfg.top_p, u)
    got = got.cpu().numpy()
    for r in range(rows):
        p = host_probs(logits[r], cfg)
        if cfg.temperature == 0.0:
            assert got[r] == host_pick(p, cfg, u[r]), r
            continue
        want, cum = host_pick(p, cfg, u[r])
        if got[r] != want:
            # only a draw at a cumulative boundary may round the other way
            lo, hi = sorted((int(got[r]), want))
            assert np.abs(cum[lo:hi + 1] - u[r]).min() < 1e-5, (r, got[r], want)


def test_sample_rejects_large_vocab():
    from woolly_b200 import WoollyError
    x = torch.zeros(1, 60000, device="cuda")
    with pytest.raises(WoollyError):
        ops.sample(x, 1.0, 0, 1.0, 0.5)


def test_decode_sample_greedy_matches_host_logits(tiny_models):
    """CudaTransformer.decode_sample (device step + device sampling, ids in,
    ids out) picks the greedy token of the logits the host path returns."""
    from woolly_b200.model import CudaTransformer, Session
    m = CudaTransformer(tiny_models["gqa_q4_0"], max_sessions=6, max_context=64, max_batch=3)
    a = [Session(m) for _ in range(3)]
    b = [Session(m) for _ in range(3)]
    prompts = [[1, 2, 3], [9, 8], [5, 6, 7, 8]]
    for sa, sb, pr in zip(a, b, prompts):
        sa.infer(pr)
        sb.infer(pr)
    ids = [11, 12, 13]
    for _ in range(4):
        host = np.stack(m.forward_sessions(a, [[i] for i in ids]))
        want = [int(np.flatnonzero(r == r.max())[-1]) for r in host]
        got = m.decode_sample(b, ids)
        assert list(got) == want
        ids = want
    for s in a + b:
        s.close()
    m.close()


def test_engine_device_sampling_matches_host(tiny_models):
    """Continuous batching with sampling on the GPU gives the same tokens as
    with the host restatement of the server's rules (same per-request
    streams), for greedy and sampled requests mixed in one batch."""
    from woolly_b200.engine import BatchEngine
    from woolly_b200.model import CudaTransformer
    rng = np.random.default_rng(5)
    prompts = [rng.integers(3, 1024, int(n)).tolist() for n in (5, 9, 3, 12)]
    cfgs = [GenerationConfig(max_tokens=8, eos_below=0, temperature=t, top_k=k, top_p=p, seed=i)
            for i, (t, k, p) in enumerate([(0.0, 0, 1.0), (0.8, 20, 1.0), (1.0, 0, 0.9),
                                           (0.7, 50, 0.95)])]
    runs = []
    for dev in (False, True):
        m = CudaTransformer(tiny_models["gqa_q4_0"], max_sessions=4, max_context=64, max_batch=4)
        eng = BatchEngine(m, device_sampling=dev)
        assert eng.device_sampling == dev
        ids = [eng.submit(p, c) for p, c in zip(prompts, cfgs)]
        eng.run()
        runs.append([eng.finished[i].tokens for i in ids])
        eng.close()
        m.close()
    assert runs[0] == runs[1]
