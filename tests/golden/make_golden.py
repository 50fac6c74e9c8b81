"""Regenerates the committed fixtures in tests/golden/.

kats.json: the reference's dequant known-answer tests
  (crates/woolly-tensor/src/quantization.rs:1294-1386), encoded as raw GGUF
  block bytes plus the expected values stated in those tests.
tiny_forward.npz: logits of the CPU oracle for a small seeded model written by
  woolly_b200's synthetic GGUF writer (spec + ids stored alongside), used to
  pin the oracle/writer pair and as a GPU parity target.

    python tests/golden/make_golden.py
"""
import json
import os
import struct
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle")]

TINY = dict(hidden=256, layers=2, heads=4, kv_heads=2, ff=512, vocab=512, weight_type=2, seed=2024)
TINY_IDS = [5, 17, 300, 2, 511, 42, 99, 256]


def kats():
    q4 = lambda d, qs: struct.pack("<e", d) + bytes(qs)
    out = [
        dict(source="quantization.rs:1294-1307", type=2, n=32, hex=q4(2.0, [0] * 16).hex(),
             expect=[-16.0] * 32),
        dict(source="quantization.rs:1310-1326", type=3, n=32,
             hex=(struct.pack("<ee", 1.0, 5.0) + bytes([1] * 16)).hex(),
             expect=[6.0] * 16 + [5.0] * 16),
        dict(source="quantization.rs:1329-1344", type=8, n=32,
             hex=(struct.pack("<e", 0.5) + bytes([10, 251] + [0] * 30)).hex(),
             expect=[5.0, -2.5] + [0.0] * 30),
        dict(source="quantization.rs:1359-1386", type=2, n=64,
             hex=(q4(1.0, [0x11] * 16) + q4(2.0, [0x22] * 16)).hex(),
             expect=[-7.0] * 32 + [-12.0] * 32),
    ]
    return {"dequant": out}


def main():
    import oracle as O
    from woolly_b200.gguf import write_synthetic
    with open(os.path.join(HERE, "kats.json"), "w") as f:
        json.dump(kats(), f, indent=1)
    with tempfile.TemporaryDirectory() as td:
        p = write_synthetic(os.path.join(td, "tiny.gguf"), **TINY)
        m = O.Model(p)
        kv = m.new_kv(64)
        logits = m.forward(kv, TINY_IDS, all_rows=True)
        m.close()
    np.savez_compressed(os.path.join(HERE, "tiny_forward.npz"), logits=logits,
                        ids=np.array(TINY_IDS, np.uint32),
                        spec=np.array(json.dumps(TINY)))
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
