"""Pin the CPU oracle to the reference's own known-answer tests.

Each test below restates one unit test of crates/kestrel-engine (same inputs,
same assertion, same tolerance) and runs it against the oracle library. The
Rust code cannot run here, so these tests are what tie the restatement to the
reference; the lane-emulation tests then tie the AVX2 kernels to the scalar
specification that the CUDA kernels reproduce.
"""
import numpy as np
import pytest

import oracle
from kestrel_b200 import ggml as G


def test_q8_0_and_q4_0_known_values():
    """quant.rs:374-394 (q8_0_and_q4_0_known_values)."""
    b = np.zeros(34, np.uint8)
    b[:2] = np.frombuffer(G.f16_bytes(0.5), np.uint8)
    b[2:] = (np.arange(32) - 16).astype(np.int8).view(np.uint8)
    y = oracle.dequant_row(G.Q8_0, b, 32)
    assert y[0] == -8.0
    assert y[31] == 7.5

    b = np.zeros(18, np.uint8)
    b[:2] = np.frombuffer(G.f16_bytes(2.0), np.uint8)
    b[2] = 0x9F
    y = oracle.dequant_row(G.Q4_0, b, 32)
    assert y[0] == 14.0
    assert y[16] == 2.0
    assert y[1] == -16.0


def test_matmul_matches_naive():
    """quant.rs:396-410 (matmul_matches_naive): F32 weights, s=3 rows."""
    rows, cols, s = 37, 64, 3
    i = np.arange(rows * cols)
    wf = (((i * 31) % 17).astype(np.float32) - 8.0) * np.float32(0.1)
    x = ((np.arange(s * cols) % 5).astype(np.float32) - 2.0)
    out = oracle.matmul(G.F32, wf.view(np.uint8), rows, cols, x.reshape(s, cols))
    e = x.reshape(s, cols).astype(np.float64) @ wf.reshape(rows, cols).astype(np.float64).T
    assert np.all(np.abs(out - e) < 1e-3)


def _blocks(t, n, seed, scale):
    """qdot.rs:275-299 / avx2.rs:198-208: xorshift bytes, then f16 scales."""
    raw = G.xorshift_bytes(G.bytes_for(t, n), seed)
    return G.set_block_scales(raw, t, scale)


UNPACK_TYPES = [G.Q8_0, G.Q4_0, G.Q4_1, G.Q5_0, G.Q5_1, G.Q4_K, G.Q5_K, G.Q6_K]


@pytest.mark.parametrize("t", UNPACK_TYPES, ids=[G.NAMES[t] for t in UNPACK_TYPES])
def test_unpack_matches_dequantization_exactly(t):
    """qdot.rs:301-315: unpack == dequant_row within 1e-5*max(|w|,1)."""
    n = 1024
    w = _blocks(t, n, 7, 0.01)
    wf = oracle.dequant_row(t, w, n)
    q, sc, mn = oracle.unpack(t, w, n)
    v = sc[np.arange(n) // 16] * q.astype(np.float32) - mn[np.arange(n) // 16]
    assert np.all(np.abs(v - wf) <= 1e-5 * np.maximum(np.abs(wf), 1.0))


@pytest.mark.parametrize("t", [G.Q8_0, G.Q4_K, G.Q6_K, G.Q5_1], ids=["Q8_0", "Q4_K", "Q6_K", "Q5_1"])
def test_dot_close_to_float(t):
    """qdot.rs:317-333: int8 dot vs float dot within the quantisation bound."""
    n = 1024
    x = (((np.arange(n) * 37) % 101).astype(np.float32) - 50.0) / np.float32(25.0)
    q, d, s16 = oracle.q8_quantize(x)
    w = _blocks(t, n, 3, 0.01)
    wf = oracle.dequant_row(t, w, n)
    exact = oracle.dot(wf, x)
    uq, usc, umn = oracle.unpack(t, w, n)
    fast = oracle.dot_unpacked(uq, usc, umn, q, d, s16)
    tol = float(np.abs(wf).sum(dtype=np.float32)) * 2.0 / 127.0 * 0.6
    assert abs(exact - fast) <= max(tol, 1e-3)


@pytest.mark.parametrize("t", [G.Q8_0, G.Q4_0, G.Q4_K, G.Q6_K], ids=["Q8_0", "Q4_0", "Q4_K", "Q6_K"])
def test_fused_kernels_match_unpacked_reference(t):
    """avx2.rs:184-223: fused and generic kernels vs the scalar reference, 1e-4."""
    n = 2048
    x = (((np.arange(n) * 53) % 211).astype(np.float32) - 105.0) / np.float32(40.0)
    q, d, s16 = oracle.q8_quantize(x)
    w = _blocks(t, n, 9, 0.02)
    uq, usc, umn = oracle.unpack(t, w, n)
    # The reference's scalar loop (avx2.rs:212-216) is dot_impl's order.
    r = oracle.dot_unpacked(uq, usc, umn, q, d, s16, scalar=True)
    fused = oracle.dot_fused(t, w, q, d, s16)
    generic = oracle.dot_unpacked(uq, usc, umn, q, d, s16)
    tol = 1e-4 * max(abs(r), 1.0)
    assert abs(fused - r) <= tol
    assert abs(generic - r) <= tol


@pytest.mark.parametrize("shape", [(7, 9, 64), (3, 4, 8), (1, 1, 24), (10, 3, 256)])
def test_gemm_matches_naive(shape):
    """avx2.rs:310-330 (gemm_matches_naive)."""
    rows, s_rows, cols = shape
    w = ((((np.arange(rows * cols) * 7) % 13).astype(np.float32)) - 6.0) * np.float32(0.1)
    x = ((((np.arange(s_rows * cols) * 5) % 11).astype(np.float32)) - 5.0) * np.float32(0.2)
    res = oracle.gemm_f32(w, rows, x, s_rows, cols)
    e = w.reshape(rows, cols).astype(np.float64) @ x.reshape(s_rows, cols).astype(np.float64).T
    assert np.all(np.abs(res - e) < 1e-3)


@pytest.mark.parametrize("t", [G.Q4_K, G.Q6_K], ids=["Q4_K", "Q6_K"])
def test_q8k_kernels_match_dequantized_math(t):
    """avx2.rs:421-460: Q8_K kernels vs f64 sum of dequantised values, 1e-3."""
    n = 2048
    x = (((np.arange(n) * 53) % 211).astype(np.float32) - 105.0) / np.float32(40.0)
    q, d, bs = oracle.q8k_quantize(x)
    w = _blocks(t, n, 7, 0.02)
    uq, usc, umn = oracle.unpack(t, w, n)
    i = np.arange(n)
    wv = (usc[i // 16] * uq.astype(np.float32) - umn[i // 16]).astype(np.float64)
    r = float(np.sum(wv * q.astype(np.float64) * d[i // 256].astype(np.float64)))
    got = oracle.dot_fused_k(t, w, q, d, bs)
    assert abs(got - r) <= 1e-3 * max(abs(r), 1.0)


# ---------------------------------------------------------------------------
# Lane emulation == AVX2, bit for bit (the specification the GPU follows).

def _seeded_row(t, n, seed):
    rng = np.random.default_rng(seed)
    w = rng.integers(0, 256, G.bytes_for(t, n), dtype=np.uint8)
    return G.set_block_scales(w, t, 0.013)


@pytest.mark.parametrize("t", [G.Q4_K, G.Q6_K], ids=["Q4_K", "Q6_K"])
@pytest.mark.parametrize("n", [256, 768, 2048, 14336])
def test_q8k_lane_emulation_bit_exact(t, n):
    rng = np.random.default_rng(n + t)
    for trial in range(6):
        x = rng.standard_normal(n).astype(np.float32) * np.float32(1 + trial)
        q, d, bs = oracle.q8k_quantize(x)
        w = _seeded_row(t, n, 100 * trial + n)
        a = oracle.dot_fused_k(t, w, q, d, bs)
        b = oracle.dot_fused_k(t, w, q, d, bs, lanes=True)
        assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)


def test_q8_0_lane_emulation_bit_exact():
    rng = np.random.default_rng(5)
    for n in (32, 512, 4096):
        x = rng.standard_normal(n).astype(np.float32)
        q, d, s16 = oracle.q8_quantize(x)
        w = _seeded_row(G.Q8_0, n, n)
        a = oracle.dot_fused(G.Q8_0, w, q, d, s16)
        b = oracle.dot_q8_0_lanes(w, q, d)
        assert np.float32(a).view(np.uint32) == np.float32(b).view(np.uint32)


def test_gemm_lanes_match_scalar_chain():
    """gemm_f32's 3x4 blocked outputs equal the 8-lane FMA chain + hsum, and its
    remainder rows/columns equal dot_f32."""
    rng = np.random.default_rng(11)
    rows, s_rows, cols = 8, 6, 64
    w = rng.standard_normal(rows * cols).astype(np.float32)
    x = rng.standard_normal(s_rows * cols).astype(np.float32)
    res = oracle.gemm_f32(w, rows, x, s_rows, cols)
    W, X = w.reshape(rows, cols), x.reshape(s_rows, cols)
    for r in range(rows):
        for s in range(s_rows):
            blocked = r < rows // 3 * 3 and s < s_rows // 4 * 4
            e = oracle.lane_chain_f32(W[r], X[s]) if blocked else oracle.dot_f32(W[r], X[s])
            assert np.float32(res[r, s]).view(np.uint32) == np.float32(e).view(np.uint32)


def test_q8k_quantize_rules():
    """Q8KRow::quantize (qdot.rs:347-367): d = amax/127, round half away from
    zero, clamp +-127, bsums per 16; all-zero blocks give d = 0 and q = 0."""
    x = np.zeros(512, np.float32)
    x[:256] = np.linspace(-3, 3, 256, dtype=np.float32)
    x[5] = 0.5 * (3.0 / 127.0) * 3  # lands near a .5 boundary after scaling
    q, d, bs = oracle.q8k_quantize(x)
    amax = np.abs(x[:256]).max()
    assert d[0] == np.float32(amax) / np.float32(127)
    assert d[1] == 0 and np.all(q[256:] == 0)
    inv = np.float32(1) / d[0]
    v = x[:256] * inv
    ref = np.clip(np.sign(v) * np.floor(np.abs(v) + np.float32(0.5)), -127, 127).astype(np.int8)
    assert np.array_equal(q[:256], ref)
    assert np.array_equal(bs, q.reshape(-1, 16).astype(np.int32).sum(axis=1))
