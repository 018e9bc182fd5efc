"""Committed golden fixtures vs the oracle and the quantizer (CPU only)."""
import os

import numpy as np
import pytest

import oracle
from kestrel_b200 import ggml as G

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def deq():
    return np.load(os.path.join(HERE, "dequant_gguf.npz"))


@pytest.mark.parametrize("name", ["Q4_K", "Q6_K", "Q8_0", "Q4_0"])
def test_oracle_decode_matches_gguf_py(deq, name):
    """Block decoding equals gguf-py's independent decoder bit for bit."""
    t = G.BY_NAME[name]
    w, ref = deq[f"{name}_bytes"], deq[f"{name}_f32"]
    got = oracle.dequant(t, w, w.shape[0], ref.shape[1])
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_moe_fixture_reproduced():
    fx = np.load(os.path.join(HERE, "moe_small.npz"))
    k, ff = int(fx["k"]), int(fx["ff"])
    for n in (1, 3, 4, 9):
        o, ids, w = oracle.moe_ffn(fx[f"h{n}"], fx["router"], k, G.Q4_K, fx["gate"], G.Q4_K, fx["up"],
                                   G.Q6_K, fx["down"], ff)
        assert np.array_equal(ids, fx[f"ids{n}"])
        assert np.array_equal(w.view(np.uint32), fx[f"w{n}"].view(np.uint32))
        assert np.array_equal(o.view(np.uint32), fx[f"out{n}"].view(np.uint32))


def test_quantizer_stable():
    """The fixture's Q4_K/Q6_K bytes come from this quantizer with seed 77."""
    fx = np.load(os.path.join(HERE, "moe_small.npz"))
    rng = np.random.default_rng(77)
    E, d, ff = int(fx["E"]), int(fx["d"]), int(fx["ff"])
    gate = G.quantize(G.Q4_K, rng.standard_normal((E * ff, d)).astype(np.float32) * 0.02)
    up = G.quantize(G.Q4_K, rng.standard_normal((E * ff, d)).astype(np.float32) * 0.02)
    down = G.quantize(G.Q6_K, rng.standard_normal((E * d, ff)).astype(np.float32) * 0.02)
    assert np.array_equal(gate, fx["gate"]) and np.array_equal(up, fx["up"]) and np.array_equal(down, fx["down"])


@pytest.mark.parametrize("t", [G.Q4_K, G.Q6_K, G.Q8_0])
def test_quantizer_error_bounded(t):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((8, 1024)).astype(np.float32) * 0.02
    y = oracle.dequant(t, G.quantize(t, x), 8, 1024)
    rel = np.abs(y - x).max() / np.abs(x).max()
    assert rel < {G.Q4_K: 0.08, G.Q6_K: 0.03, G.Q8_0: 0.006}[t]
