import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


@pytest.fixture(scope="session")
def tiny_models(tmp_path_factory):
    """Small seeded GGUF models written by the library's synthetic writer."""
    from woolly_b200.gguf import write_synthetic
    from woolly_b200 import Q4_0, Q4_1, Q8_0
    d = tmp_path_factory.mktemp("models")
    specs = {
        # TinyLlama-like GQA (4 q heads per kv head), head_dim 64
        "gqa_q4_0": dict(hidden=512, layers=2, heads=8, kv_heads=2, ff=768, vocab=1024,
                         weight_type=Q4_0, seed=11),
        "mha_q4_1": dict(hidden=256, layers=2, heads=2, kv_heads=2, ff=512, vocab=512,
                         weight_type=Q4_1, seed=12),
        "gqa_q8_0": dict(hidden=512, layers=2, heads=4, kv_heads=1, ff=1024, vocab=768,
                         weight_type=Q8_0, seed=13),
        # tied output (no output.weight): LM head reads the f32 embedding
        "tied_q4_0": dict(hidden=256, layers=1, heads=4, kv_heads=2, ff=256, vocab=512,
                          weight_type=Q4_0, tied=True, seed=14),
        # sliding window in metadata (Mistral shape in miniature)
        "swa_q4_1": dict(hidden=256, layers=2, heads=4, kv_heads=2, ff=512, vocab=512,
                         weight_type=Q4_1, sliding_window=16, seed=15),
    }
    out = {}
    for name, kw in specs.items():
        out[name] = write_synthetic(str(d / f"{name}.gguf"), **kw)
    return out
