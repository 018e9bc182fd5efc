"""Regenerate the committed golden fixtures (run in the build container).

* dequant_gguf.npz -- block bytes of each type with gguf-py 0.19's independent
  decoder output (`gguf.quants.dequantize`, the cross-check Kestrel's own
  fixture tool uses, tools/make_fixtures.py:193-217). Pins the oracle's and
  the GPU's block decoding to a third-party implementation.
* moe_small.npz -- a small seeded MoE layer (Q4_K gate/up, Q6_K down, F32
  router) with the oracle's outputs (layer output, top-k ids and weights) for
  several token counts, so a change to the oracle or the quantizer shows up as
  a fixture mismatch.

Usage: python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from kestrel_b200 import ggml as G  # noqa: E402


def dequant_fixture():
    from gguf import GGMLQuantizationType as QT
    from gguf import quants
    rng = np.random.default_rng(1234)
    out = {}
    for t, qt in [(G.Q4_K, QT.Q4_K), (G.Q6_K, QT.Q6_K), (G.Q8_0, QT.Q8_0), (G.Q4_0, QT.Q4_0)]:
        rows, cols = 4, 512
        # Half the rows from the quantizer, half random bytes with sane scales.
        wq = G.quantize(t, rng.standard_normal((rows // 2, cols)).astype(np.float32) * 0.02)
        wr = G.set_block_scales(rng.integers(0, 256, (rows // 2) * G.bytes_for(t, cols), dtype=np.uint8), t, 0.01)
        w = np.concatenate([wq.reshape(-1), wr]).reshape(rows, -1)
        out[f"{G.NAMES[t]}_bytes"] = w
        out[f"{G.NAMES[t]}_f32"] = quants.dequantize(w, qt).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "dequant_gguf.npz"), **out)


def moe_fixture():
    rng = np.random.default_rng(77)
    E, k, d, ff = 4, 2, 256, 256
    gate = G.quantize(G.Q4_K, rng.standard_normal((E * ff, d)).astype(np.float32) * 0.02)
    up = G.quantize(G.Q4_K, rng.standard_normal((E * ff, d)).astype(np.float32) * 0.02)
    down = G.quantize(G.Q6_K, rng.standard_normal((E * d, ff)).astype(np.float32) * 0.02)
    router = (rng.standard_normal((E, d)) * 0.02).astype(np.float32)
    fx = dict(E=E, k=k, d=d, ff=ff, gate=gate, up=up, down=down, router=router)
    for n in (1, 3, 4, 9):
        h = rng.standard_normal((n, d)).astype(np.float32)
        o, ids, w = oracle.moe_ffn(h, router, k, G.Q4_K, gate, G.Q4_K, up, G.Q6_K, down, ff)
        fx[f"h{n}"], fx[f"out{n}"], fx[f"ids{n}"], fx[f"w{n}"] = h, o, ids, w
    np.savez_compressed(os.path.join(HERE, "moe_small.npz"), **fx)


if __name__ == "__main__":
    dequant_fixture()
    moe_fixture()
    for f in sorted(os.listdir(HERE)):
        print(f, os.path.getsize(os.path.join(HERE, f)))
