"""Parity at the benchmarked shapes (GPU): the launches bench.py times, checked
against the CPU oracle with the north_star bar (teacher-forced logits max-abs
<= 1e-2, top-1 agreement >= 99%).

* LLaMA-2-7B shape: d 4096, 32 heads MHA (hd 128), FFN
  11008, vocab 32000, Q4_0, truncated to 2 of its 32 layers so the oracle
  finishes.  16 sessions x 512-token prompts (the tcgen05 prefill GEMM at
  M = 512), then teacher-forced decode at batch 16 through the device-pointer
  step the bench times, issued back to back without host synchronisation as
  the bench does (B = 16 decode GEMV; 512 (KV head, row) pairs, so the paged
  attention runs one-page rounds with context splits and the combine kernel),
  then batch-1 steps.
* Mistral-7B shape: d 4096, 32 heads, 8 KV heads, FFN
  14336, Q4_1, sliding window 4096, 1 layer; 8 sessions whose contexts run
  past the window (4,200+ tokens, prefilled in 1024-token chunks), then
  batch-8 decode.

Each test prints its measured max-abs error and top-1 agreement.
"""
import time

import numpy as np
import pytest

import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from woolly_b200 import Q4_0, Q4_1  # noqa: E402
from woolly_b200.gguf import write_synthetic  # noqa: E402
from woolly_b200.model import CudaTransformer, Session  # noqa: E402

LOGIT_TOL = 1e-2
TOP1_MIN = 0.99


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def measure(got, ref):
    got = np.asarray(got, np.float32).reshape(ref.shape)
    V = ref.shape[-1]
    err = float(np.abs(got - ref).max())
    top1 = float(np.mean(got.reshape(-1, V).argmax(-1) == ref.reshape(-1, V).argmax(-1)))
    return err, top1


def check(what, got, ref):
    err, top1 = measure(got, ref)
    print(f"{what}: max-abs {err:.3e}, top-1 {top1:.4f}, |ref| max {np.abs(ref).max():.2f}")
    assert err <= LOGIT_TOL, f"{what}: max-abs {err}"
    assert top1 >= TOP1_MIN, f"{what}: top-1 agreement {top1}"


def device_steps(m, sess, forced):
    """Decode steps through wl_decode_step_device (device ids and logits),
    queued back to back with no synchronisation in between, as bench.py
    times them."""
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    V = m.vocab_size()
    ids = torch.from_numpy(np.ascontiguousarray(forced).astype(np.int32)).to(dev)
    out = torch.empty(forced.shape[0], len(sess), V, device=dev)
    torch.cuda.synchronize()
    for t in range(forced.shape[0]):
        m.decode_step_device(sess, ids[t].data_ptr(), out[t].data_ptr(), stream)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_7b_shape_bench_config(tmp_path):
    B, P, steps, steps1 = 16, 512, 8, 4
    p = write_synthetic(str(tmp_path / "llama7b_2l.gguf"), hidden=4096, layers=2, heads=32,
                        kv_heads=32, ff=11008, vocab=32000, weight_type=Q4_0, seed=7)
    rng = np.random.default_rng(7 + 1_000_000)
    prompts = [rng.integers(0, 32000, P).tolist() for _ in range(B)]
    forced = rng.integers(0, 32000, (steps, B)).astype(np.uint32)
    forced1 = rng.integers(0, 32000, (steps1, 1)).astype(np.uint32)

    m = CudaTransformer(p, max_sessions=B, max_context=P + steps + steps1 + 8, max_batch=B,
                        max_prefill=P)
    sess = [Session(m) for _ in range(B)]
    g_pre = np.stack([s.infer_last(pr) for s, pr in zip(sess, prompts)])
    g_dec = device_steps(m, sess, forced)
    g_dec1 = device_steps(m, sess[:1], forced1)
    for s in sess:
        s.close()
    m.close()

    t0 = time.time()
    om = O.Model(p)
    kvs = [om.new_kv(P + steps + steps1 + 8) for _ in range(B)]
    o_pre = np.stack([om.forward(kv, pr, all_rows=False)[0] for kv, pr in zip(kvs, prompts)])
    o_dec = np.stack([om.decode_batch(kvs, forced[t]) for t in range(steps)])
    o_dec1 = np.stack([om.decode_batch(kvs[:1], forced1[t]) for t in range(steps1)])
    om.close()
    print(f"oracle: {time.time() - t0:.1f} s")
    check("7B shape, prefill 16 x 512 (last rows)", g_pre, o_pre)
    check("7B shape, bs16 decode", g_dec, o_dec)
    check("7B shape, bs1 decode", g_dec1, o_dec1)


def test_mistral_shape_long_context_window(tmp_path):
    B, W, steps = 8, 4096, 4
    p = write_synthetic(str(tmp_path / "mistral_1l.gguf"), hidden=4096, layers=1, heads=32,
                        kv_heads=8, ff=14336, vocab=32000, weight_type=Q4_1,
                        sliding_window=W, context_length=8192, seed=9)
    rng = np.random.default_rng(9 + 1_000_000)
    lens = rng.integers(W + 104, W + 260, B)
    prompts = [rng.integers(0, 32000, int(n)).tolist() for n in lens]
    forced = rng.integers(0, 32000, (steps, B)).astype(np.uint32)
    max_ctx = int(lens.max()) + steps + 8

    m = CudaTransformer(p, max_sessions=B, max_context=max_ctx, max_batch=B, max_prefill=1024)
    sess = [Session(m) for _ in range(B)]
    g_pre = np.stack([s.infer_last(pr) for s, pr in zip(sess, prompts)])
    g_dec = device_steps(m, sess, forced)
    for s in sess:
        s.close()
    m.close()

    t0 = time.time()
    om = O.Model(p, window=W)
    kvs = [om.new_kv(max_ctx) for _ in range(B)]
    o_pre = np.stack([om.forward(kv, pr, all_rows=False)[0] for kv, pr in zip(kvs, prompts)])
    o_dec = np.stack([om.decode_batch(kvs, forced[t]) for t in range(steps)])
    om.close()
    print(f"oracle: {time.time() - t0:.1f} s")
    check("Mistral shape, prefill past the window (last rows)", g_pre, o_pre)
    check("Mistral shape, bs8 decode at context > window", g_dec, o_dec)
