"""Greedy decode of several independent sequences in lockstep (run with -m gpu):
kc_model_generate_batch through the C ABI against the oracle's batch-1
Engine::generate (crates/kestrel-engine/src/lib.rs:98-166 with
SamplerConfig::greedy) of every prompt alone.

The reference serves one sequence per Engine, so a batch of 8 is 8 such runs.
On the GPU a step carries one row per sequence, and each row must come out
as a batch of one: the router's sums in quant::dot order (not gemm_f32's,
which quant::matmul picks for 4 or more rows), every expert and dense product
on the int8 path (experts chosen by 4 or more sequences are split into
entries of at most three rows), attention over the row's own cache at its
own position. Prompts are evaluated with the reference's exact f32 order
(KC_OPT_F32_PREFILL), so every sequence's tokens must equal the oracle's.
"""
import numpy as np
import pytest

import oracle
from kestrel_b200 import ggml as G
from kestrel_b200 import synth

from gpu_util import oracle_model

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def ctx():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from kestrel_b200.cuda import Context
    c = Context(0)
    yield c
    c.close()


def prompts_of(cfg, lens, seed):
    rng = np.random.default_rng(seed)
    return [[int(t) for t in rng.integers(0, cfg["n_vocab"], n)] for n in lens]


def run_batch(ctx, model, prompts, n_gen, n_ctx):
    from kestrel_b200.cuda import OPT_F32_PREFILL
    ctx.set_option(OPT_F32_PREFILL, 1)
    try:
        synth.load_cuda(ctx, model, n_ctx=n_ctx)
        return ctx.model_generate_batch(prompts, n_gen)
    finally:
        ctx.set_option(OPT_F32_PREFILL, 0)


def oracle_tokens(model, prompts, n_gen, n_ctx):
    out = []
    for p in prompts:
        toks, _ = oracle_model(oracle, model, n_ctx=n_ctx).generate(p, n_gen)
        out.append(toks)
    return out


def first_diff(a, b):
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), None)


def test_batch8_config0_matches_oracle(ctx):
    """configs[0]'s model (8 experts, top-2): 8 sequences with prompts of 1 to
    37 tokens (the 1-3 token prompts take the int8 path, the others the f32
    one), 16 greedy tokens each. With 16 selections over 8 experts per step,
    experts regularly get 4 or more rows."""
    model = synth.make_model(synth.CONFIG0, seed=0)
    cfg = model["cfg"]
    prompts = prompts_of(cfg, [1, 3, 5, 8, 13, 21, 30, 37], seed=21)
    got = run_batch(ctx, model, prompts, 16, n_ctx=64)
    ref = oracle_tokens(model, prompts, 16, n_ctx=64)
    bad = [(s, first_diff(g, r)) for s, (g, r) in enumerate(zip(got, ref)) if g != r]
    assert not bad, bad


def test_batch_equals_single_sequence_runs(ctx):
    """The same model and prompts through kc_model_generate one at a time and
    through one batch of 5 and one of 8: identical tokens (a sequence's
    tokens do not depend on its batch)."""
    from kestrel_b200.cuda import OPT_F32_PREFILL
    model = synth.make_model(synth.CONFIG0, seed=0)
    prompts = prompts_of(model["cfg"], [9, 2, 17, 4, 11, 6, 25, 1], seed=22)
    ctx.set_option(OPT_F32_PREFILL, 1)
    try:
        synth.load_cuda(ctx, model, n_ctx=64)
        single = []
        for p in prompts:
            ctx.model_truncate(0)
            single.append(ctx.model_generate(p, 20))
        b5 = ctx.model_generate_batch(prompts[:5], 20)
        b8 = ctx.model_generate_batch(prompts, 20)
        # sequence 0 is the single-sequence calls' cache: its prompt and 19 steps
        assert ctx.model_cached() == len(prompts[0]) + 19
        # a single sequence again after the batches
        ctx.model_truncate(0)
        again = ctx.model_generate(prompts[2], 20)
    finally:
        ctx.set_option(OPT_F32_PREFILL, 0)
    assert b5 == single[:5]
    assert b8 == single
    assert again == single[2]


def test_decode_continues_across_calls(ctx):
    """kc_model_prefill_seq per sequence, then kc_model_decode_seqs twice (8,
    then 9 tokens: the second call starts from the first call's last token)
    gives the tokens of one 16-token kc_model_generate per prompt."""
    from kestrel_b200.cuda import OPT_F32_PREFILL
    model = synth.make_model(synth.CONFIG0, seed=0)
    prompts = prompts_of(model["cfg"], [6, 2, 14], seed=24)
    ctx.set_option(OPT_F32_PREFILL, 1)
    try:
        synth.load_cuda(ctx, model, n_ctx=48)
        single = []
        for p in prompts:
            ctx.model_truncate(0)
            single.append(ctx.model_generate(p, 16))
        ctx.model_set_sequences(3)
        firsts = [ctx.model_prefill_seq(s, p) for s, p in enumerate(prompts)]
        a = ctx.model_decode_seqs(3, 8)
        b = ctx.model_decode_seqs(3, 9)
    finally:
        ctx.set_option(OPT_F32_PREFILL, 0)
    assert firsts == [t[0] for t in single]
    for s in range(3):
        assert [r for r in a[s]] + b[s][1:] == single[s], s
        assert b[s][0] == a[s][-1]


def test_batch8_qwen3_30b_shape_family(ctx):
    """configs[3]'s layer family at reduced size (head_dim 128, 4:1 GQA, Q4_K
    attention and embedding, Q6_K head, 16 experts top-4 Q4_K/Q6_K): 8
    sequences, 16 greedy tokens each, equal to the same prompts decoded one at
    a time on the GPU, and the first token of each equal to the oracle's."""
    from kestrel_b200.cuda import OPT_F32_PREFILL
    cfg = dict(synth.CONFIG0, n_layer=2, d=1024, n_head=8, n_kv=2, head_dim=128, rope_dim=128, rope_base=1e6,
               n_vocab=2048, n_expert=16, k=4, ff=512, t_attn=G.Q4_K, t_embd=G.Q4_K, t_out=G.Q6_K, t_gate=G.Q4_K,
               t_down=G.Q6_K)
    model = synth.make_model(cfg, seed=13)
    prompts = prompts_of(cfg, [40, 7, 3, 19, 28, 1, 12, 33], seed=23)
    got = run_batch(ctx, model, prompts, 16, n_ctx=64)
    ctx.set_option(OPT_F32_PREFILL, 1)
    try:
        single = []
        for p in prompts:
            ctx.model_truncate(0)
            single.append(ctx.model_generate(p, 16))
    finally:
        ctx.set_option(OPT_F32_PREFILL, 0)
    assert got == single
    for s, p in enumerate(prompts):
        toks, _ = oracle_model(oracle, model, n_ctx=64).generate(p, 1)
        assert got[s][0] == toks[0], s


def test_batch_errors(ctx):
    from kestrel_b200.cuda import KestrelCudaError
    model = synth.make_model(synth.CONFIG0, seed=0)
    synth.load_cuda(ctx, model, n_ctx=16)
    with pytest.raises(KestrelCudaError) as e:
        ctx.model_generate_batch([[1, 2, 3]] * 33, 2)  # more than 32 sequences
    assert e.value.code == 1
    with pytest.raises(KestrelCudaError) as e:
        ctx.model_generate_batch([[1] * 10, [2] * 12], 6)  # 12 + 5 positions > n_ctx 16
    assert e.value.code == 1
    with pytest.raises(KestrelCudaError) as e:
        ctx.model_generate_batch([[1], []], 2)  # empty prompt
    assert e.value.code == 1
    ctx.model_set_sequences(2)
    ctx.model_prefill_seq(0, [1, 2])
    with pytest.raises(KestrelCudaError) as e:
        ctx.model_decode_seqs(2, 2)  # sequence 1 has no prompt
    assert e.value.code == 7
    ctx.model_forward([5])
    with pytest.raises(KestrelCudaError) as e:
        ctx.model_decode_seqs(1, 2)  # sequence 0 was moved on by kc_model_forward
    assert e.value.code == 7
