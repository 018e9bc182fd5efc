"""GPU parity of the building blocks against the CPU oracle (run with -m gpu).

Bit-exact: Q8_K / Q8 activation quantisation, per-superblock integer sums,
router logits, top-k ids, and the int8 dequant-dot matvec (n < 4 rows), whose
float operation order reproduces the reference's AVX2 lanes. Tolerance
(1e-3 * max(max|ref|, 1), the reference's convention): the f32 path (n >= 4).
"""
import numpy as np
import pytest

import oracle
from kestrel_b200 import ggml as G

from gpu_util import bits, tol_ok

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kestrel_b200.cuda import Context
    c = Context(0)
    # Share torch's stream so the tests' host->device copies are ordered with
    # the library's kernels.
    c.set_stream(torch.cuda.current_stream().cuda_stream)
    yield c
    c.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _act_rows(rng, n, cols):
    x = rng.standard_normal((n, cols)).astype(np.float32)
    x[0, :256] *= 0  # an all-zero block (d = 0)
    if n > 1:
        x[1, :32] = 1e-30  # tiny values
        x[1, 32:64] = np.float32(127.0 / 2) * np.arange(32, dtype=np.float32) / 63  # .5 boundaries
    return x


@pytest.mark.parametrize("cols", [256, 2048, 4096])
def test_q8k_quantize_bit_exact(ctx, cols):
    rng = np.random.default_rng(cols)
    x = _act_rows(rng, 5, cols)
    q = torch.empty((5, cols), dtype=torch.int8, device="cuda")
    d = torch.empty((5, cols // 256), dtype=torch.float32, device="cuda")
    bs = torch.empty((5, cols // 16), dtype=torch.int32, device="cuda")
    ctx.q8k_quantize_dev(dev(x), q, d, bs)
    for r in range(5):
        rq, rd, rbs = oracle.q8k_quantize(x[r])
        assert np.array_equal(host(q)[r], rq)
        assert np.array_equal(bits(host(d)[r]), bits(rd))
        assert np.array_equal(host(bs)[r], rbs)


@pytest.mark.parametrize("cols", [32, 1408, 2048])
def test_q8_quantize_bit_exact(ctx, cols):
    rng = np.random.default_rng(cols + 1)
    x = rng.standard_normal((3, cols)).astype(np.float32)
    x[0, :32] = 0
    q = torch.empty((3, cols), dtype=torch.int8, device="cuda")
    d = torch.empty((3, cols // 32), dtype=torch.float32, device="cuda")
    s16 = torch.empty((3, cols // 16), dtype=torch.int32, device="cuda")
    ctx.q8_quantize_dev(dev(x), q, d, s16)
    for r in range(3):
        rq, rd, rs = oracle.q8_quantize(x[r])
        assert np.array_equal(host(q)[r], rq)
        assert np.array_equal(bits(host(d)[r]), bits(rd))
        assert np.array_equal(host(s16)[r], rs)


@pytest.mark.parametrize("t", [G.Q4_K, G.Q6_K], ids=["Q4_K", "Q6_K"])
def test_block_sums_bit_exact(ctx, t):
    """Per-superblock int32 lane sums and min/offset terms == the reference's
    AVX2 lanes (oracle lane emulation, itself checked bit-exact vs AVX2)."""
    rng = np.random.default_rng(t)
    rows, cols, n_act = 5, 1024, 2
    w = G.set_block_scales(rng.integers(0, 256, rows * G.bytes_for(t, cols), dtype=np.uint8), t, 0.01)
    x = rng.standard_normal((n_act, cols)).astype(np.float32)
    qs = [oracle.q8k_quantize(x[a]) for a in range(n_act)]
    q = np.stack([v[0] for v in qs])
    bs = np.stack([v[2] for v in qs])
    out = torch.empty((n_act, rows, cols // 256, 9), dtype=torch.int32, device="cuda")
    ctx.block_sums_dev(t, dev(w), rows, cols, dev(q), dev(bs), n_act, out)
    got = host(out)
    wr = w.reshape(rows, -1)
    for a in range(n_act):
        for r in range(rows):
            ref = oracle.block_sums_k(t, wr[r], q[a], bs[a])
            assert np.array_equal(got[a, r], ref)


@pytest.mark.parametrize("t,rows,cols", [
    (G.Q4_K, 768, 2048), (G.Q4_K, 100, 512), (G.Q6_K, 2048, 768), (G.Q6_K, 37, 1536),
    (G.Q8_0, 512, 512), (G.Q8_0, 130, 1408),
])
@pytest.mark.parametrize("n", [1, 2, 3])
def test_matmul_int8_path_bit_exact(ctx, t, rows, cols, n):
    """quant::matmul with n < 4 rows: Q8_K (K-quants) / Q8Row (Q8_0) path."""
    rng = np.random.default_rng(rows * 7 + cols + n)
    w = G.quantize(t, rng.standard_normal((rows, cols)).astype(np.float32) * np.float32(0.02))
    x = rng.standard_normal((n, cols)).astype(np.float32)
    tid = 1000 + t
    ctx.upload_dense(tid, t, w, rows, cols)
    got = ctx.matmul(tid, x)
    ref = oracle.matmul(t, w, rows, cols, x)
    assert np.array_equal(bits(got), bits(ref))


@pytest.mark.parametrize("t,rows,cols", [(G.Q4_K, 768, 2048), (G.Q6_K, 2048, 768), (G.Q8_0, 256, 1408)])
@pytest.mark.parametrize("n", [4, 5, 33])
def test_matmul_f32_path(ctx, t, rows, cols, n):
    """quant::matmul with n >= 4 rows: exact dequantisation + f32 products."""
    rng = np.random.default_rng(rows + cols + n)
    w = G.quantize(t, rng.standard_normal((rows, cols)).astype(np.float32) * np.float32(0.02))
    x = rng.standard_normal((n, cols)).astype(np.float32)
    ctx.upload_dense(2000 + t, t, w, rows, cols)
    got = ctx.matmul(2000 + t, x)
    ref = oracle.matmul(t, w, rows, cols, x)
    ok, err, scale = tol_ok(got, ref)
    assert ok, (err, scale)


@pytest.mark.parametrize("E,d", [(8, 512), (128, 2048), (8, 4096)])
@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 7, 8, 13, 64])
def test_router_logits_bit_exact(ctx, E, d, n):
    """F32 router matmul in the reference's order: scalar dot (n < 4), gemm_f32
    blocks and dot_f32 remainders (n >= 4)."""
    rng = np.random.default_rng(E + d + n)
    rw = (rng.standard_normal((E, d)) * 0.02).astype(np.float32)
    h = rng.standard_normal((n, d)).astype(np.float32)
    logits = torch.empty((n, E), dtype=torch.float32, device="cuda")
    ctx.router_logits_dev(dev(rw), dev(h), logits)
    ref = oracle.matmul(G.F32, rw.view(np.uint8), E, d, h)
    assert np.array_equal(bits(host(logits)), bits(ref))


@pytest.mark.parametrize("E,k", [(8, 2), (128, 8), (64, 6), (40, 4), (256, 8)])
def test_route_topk(ctx, E, k):
    """Top-k ids bit-exact; weights within a few ulps (CUDA expf vs glibc)."""
    rng = np.random.default_rng(E * k)
    n = 37
    logits = rng.standard_normal((n, E)).astype(np.float32)
    logits[0, :4] = 1.5  # exact ties -> lower index first
    logits[1, :] = -0.25  # every entry tied: ids 0 .. k-1
    logits[2, ::3] = 3.0  # ties spread over the lanes
    for norm, ws in [(True, 0.0), (False, 0.0), (True, 2.5)]:
        ids = torch.empty((n, k), dtype=torch.int32, device="cuda")
        w = torch.empty((n, k), dtype=torch.float32, device="cuda")
        ctx.route_dev(dev(logits), k, ids, w, norm, ws)
        rids, rw = oracle.route(logits, k, norm, ws)
        assert np.array_equal(host(ids), rids)
        np.testing.assert_allclose(host(w), rw, rtol=2e-6, atol=0)


@pytest.mark.parametrize("t", [G.Q4_K, G.Q6_K, G.Q8_0], ids=["Q4_K", "Q6_K", "Q8_0"])
def test_gpu_quantizer_matches_numpy(ctx, t):
    rng = np.random.default_rng(40 + t)
    x = (rng.standard_normal((6, 1024)) * 0.02).astype(np.float32)
    x[1] *= 0  # all-zero blocks
    x[2, :300] = np.abs(x[2, :300])  # non-negative blocks (min 0)
    out = torch.empty((6, G.bytes_for(t, 1024)), dtype=torch.uint8, device="cuda")
    ctx.quantize_dev(t, dev(x), out)
    got, ref = host(out), G.quantize(t, x)
    bad = np.argwhere(got != ref)
    detail = [(int(r), int(c), int(got[r, c]), int(ref[r, c])) for r, c in bad[:12]]
    assert len(bad) == 0, f"{len(bad)} bytes differ (row, byte, gpu, numpy): {detail}"


def test_errors_are_reported(ctx):
    from kestrel_b200.cuda import KestrelCudaError
    with pytest.raises(KestrelCudaError) as e:
        ctx.moe_ffn(12345, np.zeros((1, 256), np.float32), router_w=np.zeros((8, 256), np.float32), k=2)
    assert e.value.code == 7  # KC_ERR_STATE
    with pytest.raises(KestrelCudaError) as e:
        ctx.upload_dense(5, G.Q4_0, np.zeros(18, np.uint8), 1, 32)
    assert e.value.code == 3  # KC_ERR_TYPE
    with pytest.raises(KestrelCudaError) as e:
        ctx.upload_dense(5, G.Q4_K, np.zeros(144, np.uint8), 1, 200)
    assert e.value.code == 2  # KC_ERR_SHAPE
