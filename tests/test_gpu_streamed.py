"""Host-streamed experts (kc_upload_experts_streamed, run with -m gpu): a layer
whose experts stay in pinned host memory and are copied into HBM slots per
call must give the same bits as the same layer uploaded resident, on every
product path (int8 decode kernel for 1-3 rows, tcgen05 for 4 or more, the
exact f32 path under KC_OPT_F32_PREFILL), while the cache evicts, admits by
force and serves from scratch slots; the counters follow ExpertStore's
(crates/kestrel-memory/src/expert.rs:358-537); prefetches are used; and a
whole model with streamed layers and router lookahead (transformer.rs:432-436,
498-508) decodes the resident model's tokens."""
import numpy as np
import pytest

import oracle
from kestrel_b200 import ggml as G
from kestrel_b200 import synth

from gpu_util import bits, make_layer, oracle_layer, tol_ok, upload

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kestrel_b200.cuda import Context
    c = Context(0)
    yield c
    c.close()


def upload_streamed(ctx, lid, L):
    ctx.upload_experts_streamed(lid, L["E"], L["d"], L["ff"], L["t_gate"], L["gate"], L["t_gate"], L["up"],
                                L["t_down"], L["down"])
    ctx.upload_router(lid, L["router"], L["k"])


def same(ctx, a, b, h):
    out_a, ids_a, w_a = ctx.moe_ffn(a, h)
    out_b, ids_b, w_b = ctx.moe_ffn(b, h)
    assert np.array_equal(ids_a, ids_b)
    assert np.array_equal(bits(w_a), bits(w_b))
    assert np.array_equal(bits(out_a), bits(out_b)), f"n={len(h)}"
    return out_b, ids_b


def check_counters(st, slot_bytes=None):
    # every use of an expert is exactly one of hit, late, miss (expert.rs:358-424)
    assert st["hits"] + st["late"] + st["misses"] == st["requests"]
    if slot_bytes:
        assert st["bytes_read"] == st["reads"] * slot_bytes


@pytest.mark.parametrize("policy", [0, 1])
def test_streamed_layer_is_bit_identical(ctx, policy):
    """16 experts top-4 (Q4_K gate/up, Q6_K down), a cache of 10 slots plus 6
    scratch slots: calls of 1 to 256 tokens (int8 and tcgen05 products) in
    an order that makes the cache evict, fall back to scratch and force."""
    L = make_layer(E=16, k=4, d=512, ff=512, seed=11)
    upload(ctx, 1, L)
    upload_streamed(ctx, 2, L)
    ctx.expert_cache_reserve(10, 6, policy)
    rng = np.random.default_rng(5)
    uniq = 0
    for it, n in enumerate([1, 2, 3, 1, 4, 9, 1, 33, 2, 64, 3, 256, 1, 5, 128, 1]):
        h = rng.standard_normal((n, L["d"])).astype(np.float32)
        _, ids = same(ctx, 1, 2, h)
        uniq += len(np.unique(ids))
    st = ctx.expert_cache_stats()
    check_counters(st)
    assert st["requests"] == uniq
    assert st["misses"] > 0 and st["hits"] > 0 and st["scratch_loads"] + st["evictions"] > 0
    if policy == 1:  # LRU always evicts; LFRU serves cold experts from scratch
        assert st["evictions"] > 0
    assert st["capacity"] == 10 and st["scratch"] == 6


def test_streamed_exact_f32_and_oracle(ctx):
    """Under KC_OPT_F32_PREFILL the streamed layer equals the resident one bit
    for bit on the exact f32 path too, and both meet the oracle's tolerance;
    configs[0]'s expert types (Q4_K gate/up, Q8_0 down, ff = 1408)."""
    from kestrel_b200.cuda import OPT_F32_PREFILL
    L = make_layer(E=8, k=2, d=512, ff=1408, t_gate=G.Q4_K, t_down=G.Q8_0, seed=12)
    upload(ctx, 1, L)
    upload_streamed(ctx, 2, L)
    ctx.expert_cache_reserve(4, 4, 0)  # 8 slots: a call may route to all 8 experts
    rng = np.random.default_rng(6)
    ctx.set_option(OPT_F32_PREFILL, 1)
    try:
        for n in (1, 3, 6, 17, 40):
            h = rng.standard_normal((n, L["d"])).astype(np.float32)
            out, ids = same(ctx, 1, 2, h)
            r_out, r_ids, _ = oracle_layer(oracle, L, h)
            assert np.array_equal(ids, r_ids)
            ok, err, scale = tol_ok(out, r_out)
            assert ok, (n, err, scale)
    finally:
        ctx.set_option(OPT_F32_PREFILL, 0)
    check_counters(ctx.expert_cache_stats())


def test_prefetch_then_demand(ctx):
    """ExpertStore::prefetch (expert.rs:451-521): predicted experts copied on
    the copy stream; a call that routes to them counts them as used (hit or
    late) and waits for the copies it needs; output unchanged."""
    L = make_layer(E=16, k=4, d=512, ff=512, seed=13)
    upload(ctx, 1, L)
    upload_streamed(ctx, 2, L)
    ctx.expert_cache_reserve(16, 0, 1)
    h = np.random.default_rng(7).standard_normal((2, L["d"])).astype(np.float32)
    _, ids_res, _ = ctx.moe_ffn(1, h)
    routed = sorted(set(ids_res.ravel().tolist()))
    ctx.expert_prefetch(2, routed + [e for e in range(16) if e not in routed][:2])
    st0 = ctx.expert_cache_stats()
    assert st0["prefetch_issued"] == len(routed) + 2
    same(ctx, 1, 2, h)
    st = ctx.expert_cache_stats()
    assert st["prefetch_used"] == len(routed)
    assert st["misses"] == 0 and st["hits"] + st["late"] == len(routed)
    # the same call again: all hits, nothing copied
    reads = st["reads"]
    same(ctx, 1, 2, h)
    st = ctx.expert_cache_stats()
    assert st["reads"] == reads and st["hits"] >= len(routed)
    check_counters(st)
    with pytest.raises(Exception):
        ctx.expert_prefetch(1, [0])  # a resident layer
    with pytest.raises(Exception):
        ctx.expert_prefetch(2, [16])  # out of range


def test_too_few_slots_and_shape_errors(ctx):
    from kestrel_b200.cuda import KestrelCudaError
    L = make_layer(E=8, k=4, d=256, ff=256, seed=14)
    upload_streamed(ctx, 3, L)
    ctx.expert_cache_reserve(2, 1, 0)
    h = np.random.default_rng(8).standard_normal((4, L["d"])).astype(np.float32)
    with pytest.raises(KestrelCudaError) as e:
        ctx.moe_ffn(3, h)  # 4 tokens x top-4 of 8 experts: more than 3 slots
    assert e.value.code == 2
    # the failed call left nothing resident: a later call with room is right
    ctx.expert_cache_reserve(8, 0, 0)
    upload(ctx, 4, L)
    same(ctx, 4, 3, h)
    # every streamed layer shares the slots' shape
    L2 = make_layer(E=8, k=4, d=256, ff=512, seed=15)
    with pytest.raises(KestrelCudaError) as e:
        upload_streamed(ctx, 5, L2)
    assert e.value.code == 2
    with pytest.raises(KestrelCudaError) as e:
        ctx.expert_cache_reserve(0, 0, 0)
    assert e.value.code == 1


def test_replacing_a_streamed_layer(ctx):
    """Uploading new experts under a streamed layer's index drops what the
    slots held: the next calls use the new weights."""
    A = make_layer(E=8, k=2, d=256, ff=256, seed=16)
    B = make_layer(E=8, k=2, d=256, ff=256, seed=17)
    B["router"] = A["router"]
    upload(ctx, 1, A)
    upload(ctx, 2, B)
    upload_streamed(ctx, 3, A)
    h = np.random.default_rng(9).standard_normal((3, 256)).astype(np.float32)
    same(ctx, 1, 3, h)
    upload_streamed(ctx, 3, B)
    same(ctx, 2, 3, h)
    # and resident again
    upload(ctx, 3, A)
    same(ctx, 1, 3, h)


@pytest.mark.parametrize("lookahead", [1, 0])
def test_model_with_streamed_layers_decodes_same_tokens(ctx, lookahead):
    """A 4-layer configs[0]-family model with every routed layer streamed
    through 6 cache slots + 2 scratch slots (8 experts per layer, top-2):
    greedy tokens equal the resident model's; with router lookahead the
    predictions are counted and prefetched."""
    from kestrel_b200.cuda import OPT_LOOKAHEAD
    cfg = dict(synth.CONFIG0, n_layer=4)
    model = synth.make_model(cfg, seed=3)
    prompt = [int(t) for t in np.random.default_rng(31).integers(0, cfg["n_vocab"], 12)]
    synth.load_cuda(ctx, model, n_ctx=64)
    ref = ctx.model_generate(prompt, 24)
    ctx.model_truncate(0)
    ctx.set_option(OPT_LOOKAHEAD, lookahead)
    synth.load_cuda(ctx, model, n_ctx=64, streamed=True)
    ctx.expert_cache_reserve(6, 2, 0)
    got = ctx.model_generate(prompt, 24)
    assert got == ref
    st = ctx.expert_cache_stats()
    check_counters(st)
    if lookahead:
        # 23 decode steps x 3 predicted layers x (1 or 2 distinct experts)
        assert st["lookahead_predicted"] >= 23 * 3
        assert 0 < st["lookahead_correct"] <= st["lookahead_predicted"]
    else:
        assert st["lookahead_predicted"] == 0 and st["prefetch_issued"] == 0


def test_batch_decode_with_streamed_layers(ctx):
    """Independent sequences decoded in lockstep (kc_model_generate_batch,
    every row as a batch of one: experts split in entries of at most three
    rows) over a model whose routed layers are streamed through 8 cache + 8
    scratch slots, with router lookahead for the 3-row steps: the same tokens
    as the resident model's batch."""
    cfg = dict(synth.CONFIG0, n_layer=3)
    model = synth.make_model(cfg, seed=4)
    rng = np.random.default_rng(32)
    prompts = [[int(t) for t in rng.integers(0, cfg["n_vocab"], n)] for n in (5, 9, 2)]
    synth.load_cuda(ctx, model, n_ctx=48)
    ref = ctx.model_generate_batch(prompts, 12)
    synth.load_cuda(ctx, model, n_ctx=48, streamed=True)
    ctx.expert_cache_reserve(8, 8, 0)
    got = ctx.model_generate_batch(prompts, 12)
    assert got == ref
    st = ctx.expert_cache_stats()
    check_counters(st)
    assert st["lookahead_predicted"] > 0
