"""Layer parity at the full shapes of configs[2] (Mixtral-8x7B: d=4096, 8
experts, top-2, ff=14336) and configs[4] (Qwen3-235B-A22B: d=4096, 128
experts, top-8, ff=1536, Zipf-skewed routing) against the CPU oracle (run
with -m gpu). Q4_K gate/up + Q6_K down quantised from N(0, 0.02) on the GPU
with this library's quantizer, then copied to the host for the oracle.

configs[4]'s skew: the reference's router has no bias term, so the synthetic
inputs carry it -- feature 0 of every token is 1 and router column 0 holds
beta_e = -1.2 * ln(1 + rank(e)) * sigma_logit (rank: a seeded permutation),
which adds beta_e to expert e's logit, making popularity roughly Zipf s=1.2."""
import numpy as np
import pytest

import oracle
from kestrel_b200 import ggml as G

from gpu_util import tol_ok

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kestrel_b200.cuda import Context
    c = Context(0)
    c.set_stream(torch.cuda.current_stream().cuda_stream)
    yield c
    c.close()


def build(ctx, lid, E, k, d, ff, seed, zipf=False):
    g = torch.Generator(device="cuda").manual_seed(seed)
    host = {}
    for name, t, rows, cols in (("gate", G.Q4_K, E * ff, d), ("up", G.Q4_K, E * ff, d), ("down", G.Q6_K, E * d, ff)):
        x = torch.empty((rows, cols), dtype=torch.float32, device="cuda").normal_(0.0, 0.02, generator=g)
        q = torch.empty((rows, G.bytes_for(t, cols)), dtype=torch.uint8, device="cuda")
        ctx.quantize_dev(t, x, q)
        torch.cuda.synchronize()
        host[name] = q.cpu().numpy()
        del x, q
    rng = np.random.default_rng(seed)
    router = (rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    if zipf:
        sigma = 0.02 * np.sqrt(d)  # std of a router logit for N(0, 1) features
        rank = rng.permutation(E)
        router[:, 0] = (-1.2 * np.log1p(rank) * sigma).astype(np.float32)
    host["router"] = router
    ctx.upload_experts(lid, E, d, ff, G.Q4_K, host["gate"], G.Q4_K, host["up"], G.Q6_K, host["down"])
    ctx.upload_router(lid, router, k)
    torch.cuda.empty_cache()
    return host


def check(ctx, lid, host, E, k, d, ff, n, seed, zipf=False):
    h = np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32)
    if zipf:
        h[:, 0] = 1.0
    out, ids, w = ctx.moe_ffn(lid, h)
    r_out, r_ids, r_w = oracle.moe_ffn(h, host["router"], k, G.Q4_K, host["gate"], G.Q4_K, host["up"], G.Q6_K,
                                       host["down"], ff)
    assert np.array_equal(ids, r_ids)
    ok, err, scale = tol_ok(out, r_out)
    assert ok, f"n={n}: max err {err} vs scale {scale}"
    return ids


def test_config2_mixtral_shape(ctx):
    E, k, d, ff = 8, 2, 4096, 14336
    host = build(ctx, 700, E, k, d, ff, seed=2)
    for n, seed in ((1, 1), (3, 2), (8, 3)):  # int8 path; n=8 puts >= 4 rows on some experts
        check(ctx, 700, host, E, k, d, ff, n, seed)


def test_config4_skewed_routing(ctx):
    E, k, d, ff = 128, 8, 4096, 1536
    host = build(ctx, 701, E, k, d, ff, seed=4, zipf=True)
    for n, seed in ((1, 1), (4, 2)):
        check(ctx, 701, host, E, k, d, ff, n, seed, zipf=True)
    ids = check(ctx, 701, host, E, k, d, ff, 64, 3, zipf=True)
    cnt = np.sort(np.bincount(ids.reshape(-1), minlength=E))[::-1]
    # The skew shows: the most popular expert gets several times the mean load.
    assert cnt[0] >= 4 * (64 * k / E)
