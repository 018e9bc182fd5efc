"""Layer-level GPU parity: kc_moe_ffn (through the C ABI) vs the CPU oracle's
Transformer::moe_ffn restatement (run with -m gpu).

Top-k ids must be identical; the layer output must satisfy the reference's
tolerance max|d| <= 1e-3 * max(max|ref|, 1) (crates/kestrel-engine/tests/
oracle.rs:75-78 with the north-star tolerance 1e-3).
"""
import os

import numpy as np
import pytest

import oracle
from kestrel_b200 import ggml as G

from gpu_util import bits, make_layer, oracle_layer, tol_ok, upload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


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


def check_layer(ctx, layer_id, L, n, seed, norm_topk=True, ws=0.0):
    rng = np.random.default_rng(seed)
    h = rng.standard_normal((n, L["d"])).astype(np.float32)
    out, ids, w = ctx.moe_ffn(layer_id, h)
    r_out, r_ids, r_w = oracle_layer(oracle, L, h, norm_topk, ws)
    assert np.array_equal(ids, r_ids)
    np.testing.assert_allclose(w, r_w, rtol=2e-6, atol=0)
    ok, err, scale = tol_ok(out, r_out)
    assert ok, f"n={n}: max err {err} vs scale {scale}"
    return h, out


def test_golden_fixture(ctx):
    fx = np.load(os.path.join(GOLDEN, "moe_small.npz"))
    E, k, d, ff = (int(fx[x]) for x in ("E", "k", "d", "ff"))
    ctx.upload_experts(900, E, d, ff, G.Q4_K, fx["gate"], G.Q4_K, fx["up"], G.Q6_K, fx["down"])
    ctx.upload_router(900, fx["router"], k)
    for n in (1, 3, 4, 9):
        out, ids, w = ctx.moe_ffn(900, fx[f"h{n}"])
        assert np.array_equal(ids, fx[f"ids{n}"])
        ok, err, scale = tol_ok(out, fx[f"out{n}"])
        assert ok, (n, err, scale)


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 9, 33, 64])
def test_small_layer(ctx, n):
    L = make_layer(E=8, k=2, d=512, ff=512, seed=1)
    upload(ctx, 1, L)
    check_layer(ctx, 1, L, n, seed=100 + n)


def test_config0_like_layer(ctx):
    """configs[0]'s MoE block: d=512, 8 experts top-2, ff=1408 with Q4_K
    gate/up and Q8_0 down (ff % 256 != 0 rules out a K-quant down)."""
    L = make_layer(E=8, k=2, d=512, ff=1408, t_gate=G.Q4_K, t_down=G.Q8_0, seed=2)
    upload(ctx, 2, L)
    for n in (1, 2, 5, 64):
        check_layer(ctx, 2, L, n, seed=200 + n)


def test_routing_options(ctx):
    L = make_layer(E=16, k=4, d=256, ff=256, seed=3)
    for lid, (norm, ws) in enumerate([(False, 0.0), (True, 2.5), (False, 0.5)]):
        upload(ctx, 30 + lid, L, norm_topk=norm, weights_scale=ws)
        check_layer(ctx, 30 + lid, L, 6, seed=300 + lid, norm_topk=norm, ws=ws)


@pytest.fixture(scope="module")
def config1(ctx):
    """Qwen3-30B-A3B MoE layer, d=2048, 128 experts top-8, ff=768,
    Q4_K gate/up + Q6_K down from N(0, 0.02), F32 router N(0, 0.02). Weights
    are quantised on the GPU (kc_quantize_dev, identical rules to the numpy
    quantizer) and copied to the host for the oracle."""
    E, k, d, ff = 128, 8, 2048, 768
    g = torch.Generator(device="cuda").manual_seed(0)
    mats = {}
    for name, t, rows, cols in (("gate", G.Q4_K, E * ff, d), ("up", G.Q4_K, E * ff, d), ("down", G.Q6_K, E * d, ff)):
        x = torch.randn((rows, cols), generator=g, device="cuda", dtype=torch.float32) * 0.02
        out = torch.empty((rows, G.bytes_for(t, cols)), dtype=torch.uint8, device="cuda")
        ctx.quantize_dev(t, x, out)
        mats[name] = out
        del x
    router = (torch.randn((E, d), generator=g, device="cuda") * 0.02).float()
    ctx.upload_experts(10, E, d, ff, G.Q4_K, mats["gate"], G.Q4_K, mats["up"], G.Q6_K, mats["down"])
    ctx.upload_router(10, router, k)
    torch.cuda.synchronize()
    L = dict(E=E, k=k, d=d, ff=ff, t_gate=G.Q4_K, t_down=G.Q6_K, router=router.cpu().numpy(),
             gate=mats["gate"].cpu().numpy(), up=mats["up"].cpu().numpy(), down=mats["down"].cpu().numpy())
    return L


@pytest.mark.parametrize("n", [1, 16])
def test_config1_layer(ctx, config1, n):
    oracle.set_threads(os.cpu_count() or 1)
    check_layer(ctx, 10, config1, n, seed=1000 + n)


def test_device_api_matches_host_api(ctx, config1):
    rng = np.random.default_rng(7)
    h = rng.standard_normal((16, 2048)).astype(np.float32)
    out_h, ids_h, w_h = ctx.moe_ffn(10, h)
    hd = torch.from_numpy(h).cuda()
    out = torch.empty_like(hd)
    ids = torch.empty((16, 8), dtype=torch.int32, device="cuda")
    w = torch.empty((16, 8), dtype=torch.float32, device="cuda")
    ctx.moe_ffn_dev(10, hd, out, ids, w)
    ctx.sync()
    assert np.array_equal(bits(out.cpu().numpy()), bits(out_h))
    assert np.array_equal(ids.cpu().numpy(), ids_h)


def test_host_and_device_uploads_agree(ctx):
    L = make_layer(E=8, k=2, d=512, ff=512, seed=9)
    upload(ctx, 40, L)
    tg = {k: torch.from_numpy(np.ascontiguousarray(L[k])).cuda() for k in ("gate", "up", "down")}
    ctx.upload_experts(41, 8, 512, 512, G.Q4_K, tg["gate"], G.Q4_K, tg["up"], G.Q6_K, tg["down"])
    ctx.upload_router(41, torch.from_numpy(L["router"]).cuda(), 2)
    h = np.random.default_rng(1).standard_normal((5, 512)).astype(np.float32)
    a = ctx.moe_ffn(40, h)[0]
    b = ctx.moe_ffn(41, h)[0]
    assert np.array_equal(bits(a), bits(b))


def test_zero_tokens(ctx):
    L = make_layer(E=8, k=2, d=256, ff=256, seed=4)
    upload(ctx, 50, L)
    out, ids, w = ctx.moe_ffn(50, np.zeros((0, 256), np.float32))
    assert out.shape == (0, 256) and ids.shape == (0, 2)


def test_repeat_calls_identical(ctx):
    """Same inputs, same bits: no state leaks between calls."""
    L = make_layer(E=8, k=2, d=512, ff=512, seed=5)
    upload(ctx, 60, L)
    rng = np.random.default_rng(3)
    h1 = rng.standard_normal((9, 512)).astype(np.float32)
    h2 = rng.standard_normal((40, 512)).astype(np.float32)
    a = ctx.moe_ffn(60, h1)[0]
    ctx.moe_ffn(60, h2)
    b = ctx.moe_ffn(60, h1)[0]
    assert np.array_equal(bits(a), bits(b))


@pytest.mark.parametrize("with_gate", [True, False])
def test_shared_expert_layer(ctx, with_gate):
    """qwen2moe layer: routed experts (no top-k renormalisation) plus the
    always-on shared expert scaled by sigmoid(gate_inp . h)
    (transformer.rs:571-587), against the oracle at token counts on both sides
    of quant::matmul's n < 4 / n >= 4 dispatch."""
    lid = 950 + int(with_gate)
    L = make_layer(8, 4, 512, 512, seed=21)
    upload(ctx, lid, L, norm_topk=False)
    rng = np.random.default_rng(22)
    sf = 1024
    sh = dict(t_gate=G.Q4_K, t_up=G.Q4_K, t_down=G.Q6_K, ff=sf,
              gate=G.quantize(G.Q4_K, rng.standard_normal((sf, 512), dtype=np.float32) * np.float32(0.02)),
              up=G.quantize(G.Q4_K, rng.standard_normal((sf, 512), dtype=np.float32) * np.float32(0.02)),
              down=G.quantize(G.Q6_K, rng.standard_normal((512, sf), dtype=np.float32) * np.float32(0.02)),
              inp=(rng.standard_normal(512, dtype=np.float32) * np.float32(0.05)) if with_gate else None)
    ctx.upload_shared_expert(lid, sf, 512, sh["t_gate"], sh["gate"], sh["t_up"], sh["up"], sh["t_down"], sh["down"],
                             sh["inp"])
    for n in (1, 3, 4, 16):
        h = rng.standard_normal((n, 512)).astype(np.float32)
        out, ids, w = ctx.moe_ffn(lid, h)
        r_out, r_ids, r_w = oracle.moe_ffn(h, L["router"], L["k"], L["t_gate"], L["gate"], L["t_gate"], L["up"],
                                           L["t_down"], L["down"], L["ff"], norm_topk=False, shared=sh)
        assert np.array_equal(ids, r_ids)
        ok, err, scale = tol_ok(out, r_out)
        assert ok, f"n={n}: max err {err} vs scale {scale}"


def test_host_and_device_entry_points_agree(ctx):
    """The host-pointer entry point (kc_moe_ffn: copies in, runs, copies out)
    and the device-pointer one (kc_moe_ffn_dev) give identical ids and output
    bits, over a sequence of token counts that repeats shapes (cached tensor
    maps reused) and regrows the workspace (maps re-encoded)."""
    L = make_layer(E=16, k=4, d=512, ff=512, seed=21)
    upload(ctx, 960, L)
    upload(ctx, 961, make_layer(E=16, k=4, d=512, ff=512, seed=22))
    rng = np.random.default_rng(40)
    for n in (1, 2, 3, 1, 4, 9, 1, 1, 33, 2, 2, 64, 3, 1, 16, 16, 16):
        for lid in (960, 961):
            h = rng.standard_normal((n, 512)).astype(np.float32)
            out, ids, _ = ctx.moe_ffn(lid, h)
            hd = torch.from_numpy(h).cuda()
            od = torch.empty_like(hd)
            idd = torch.empty((n, 4), dtype=torch.int32, device="cuda")
            ctx.moe_ffn_dev(lid, hd, od, idd)
            torch.cuda.synchronize()
            assert np.array_equal(ids, idd.cpu().numpy()), (lid, n)
            assert np.array_equal(bits(out), bits(od.cpu().numpy())), (lid, n)
