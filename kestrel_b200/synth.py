"""Seeded synthetic models with the shapes of the benchmark configurations.

There are no checkpoints here (no network); like the reference's own
benchmarks, which only use synthetic GGUFs, weights are drawn from N(0, 0.02)
with a seeded numpy generator and quantized with this package's quantizer
(`ggml.quantize`); norms are 1.0. A model is a dict of hyper-parameters plus a
list of tensors (layer, name, ggml type, data, rows, cols) named as in GGUF
(blk.N.<name>; layer -1 for token_embd / output_norm / output), which
`load_cuda` hands to a `cuda.Context`.

CONFIG0 is configs[0]: 2 layers, d_model 512, 8 query / 2 KV heads of 64,
RoPE theta 1e4, RMSNorm eps 1e-6, vocab 4096, 8 experts top-2 with
renormalised gates, expert FFN 1408; Q4_K expert gate/up, Q8_0 attention,
embedding and output, F32 router and norms. Its Q4_K ffn_down_exps would
have rows of 1408 values, which is not a multiple of Q4_K's 256-value
superblock, so the expert down projection is Q8_0.
"""
from __future__ import annotations

import numpy as np

from . import ggml as G

ARCH_LLAMA, ARCH_QWEN2, ARCH_QWEN3 = 0, 1, 2

CONFIG0 = dict(name="tiny-moe-c0", arch=ARCH_QWEN3, n_layer=2, d=512, n_head=8, n_kv=2, head_dim=64, n_vocab=4096,
               rope_dim=64, rope_base=10000.0, eps=1e-6, n_expert=8, k=2, ff=1408, norm_topk=True,
               weights_scale=0.0, t_attn=G.Q8_0, t_embd=G.Q8_0, t_out=G.Q8_0, t_gate=G.Q4_K, t_down=G.Q8_0,
               dense_ff=0)


def make_model(cfg: dict, seed: int = 0) -> dict:
    """Seeded weights of `cfg` (see CONFIG0 for the keys). dense_ff > 0 makes
    the FFN dense instead of routed."""
    rng = np.random.default_rng(seed)
    d, nh, nkv, hd = cfg["d"], cfg["n_head"], cfg["n_kv"], cfg["head_dim"]
    tensors = []

    def w(rows, cols):
        return rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02)

    def add(layer, name, t, rows, cols, data=None):
        if data is None:
            data = w(rows, cols)
        tensors.append((layer, name, t, data if t == G.F32 else G.quantize(t, data), rows, cols))

    ones = lambda n: np.ones((1, n), np.float32)
    add(-1, "token_embd", cfg["t_embd"], cfg["n_vocab"], d)
    for l in range(cfg["n_layer"]):
        add(l, "attn_norm", G.F32, 1, d, ones(d))
        add(l, "attn_q", cfg["t_attn"], nh * hd, d)
        add(l, "attn_k", cfg["t_attn"], nkv * hd, d)
        add(l, "attn_v", cfg["t_attn"], nkv * hd, d)
        if cfg["arch"] == ARCH_QWEN2:
            add(l, "attn_q_bias", G.F32, 1, nh * hd)
            add(l, "attn_k_bias", G.F32, 1, nkv * hd)
            add(l, "attn_v_bias", G.F32, 1, nkv * hd)
        if cfg["arch"] == ARCH_QWEN3:
            add(l, "attn_q_norm", G.F32, 1, hd, ones(hd))
            add(l, "attn_k_norm", G.F32, 1, hd, ones(hd))
        add(l, "attn_output", cfg["t_attn"], d, nh * hd)
        add(l, "ffn_norm", G.F32, 1, d, ones(d))
        if cfg.get("dense_ff", 0):
            f = cfg["dense_ff"]
            add(l, "ffn_gate", cfg["t_gate"], f, d)
            add(l, "ffn_up", cfg["t_gate"], f, d)
            add(l, "ffn_down", cfg["t_down"], d, f)
        else:
            E, ff = cfg["n_expert"], cfg["ff"]
            add(l, "ffn_gate_inp", G.F32, E, d)
            add(l, "ffn_gate_exps", cfg["t_gate"], E * ff, d)
            add(l, "ffn_up_exps", cfg["t_gate"], E * ff, d)
            add(l, "ffn_down_exps", cfg["t_down"], E * d, ff)
    add(-1, "output_norm", G.F32, 1, d, ones(d))
    add(-1, "output", cfg["t_out"], cfg["n_vocab"], d)
    return dict(cfg=dict(cfg), tensors=tensors)


# kc_model_tensor kinds by GGUF name.
DENSE_KINDS = {"attn_norm": 0, "attn_q": 1, "attn_k": 2, "attn_v": 3, "attn_output": 4, "attn_q_bias": 5,
               "attn_k_bias": 6, "attn_v_bias": 7, "attn_q_norm": 8, "attn_k_norm": 9, "ffn_norm": 10,
               "ffn_gate": 11, "ffn_up": 12, "ffn_down": 13}
MODEL_KINDS = {"token_embd": 0, "output_norm": 1, "output": 2}


def load_cuda(ctx, model: dict, n_ctx: int, block=None, streamed=False) -> None:
    """Declare `model` on a cuda.Context and upload its tensors (with an
    expert block, only that block of each routed layer's experts; streamed:
    the routed experts stay in host memory, kc_upload_experts_streamed)."""
    c = model["cfg"]
    ctx.model_init(c["n_layer"], c["d"], c["n_head"], c["n_kv"], c["head_dim"], c["n_vocab"], n_ctx, c["rope_dim"],
                   c["rope_base"], c["eps"], c["arch"])
    by = {}
    for layer, name, t, data, rows, cols in model["tensors"]:
        by[(layer, name)] = (t, data, rows, cols)
        if layer < 0:
            ctx.model_tensor(-1, MODEL_KINDS[name], t, data, rows, cols)
        elif name in DENSE_KINDS:
            ctx.model_tensor(layer, DENSE_KINDS[name], t, data, rows, cols)
    for l in range(c["n_layer"]):
        if (l, "ffn_gate_inp") not in by:
            continue
        tg, gate, _, _ = by[(l, "ffn_gate_exps")]
        tu, up, _, _ = by[(l, "ffn_up_exps")]
        td, down, _, _ = by[(l, "ffn_down_exps")]
        if streamed:
            ctx.upload_experts_streamed(l, c["n_expert"], c["d"], c["ff"], tg, gate, tu, up, td, down)
        elif block is None:
            ctx.upload_experts(l, c["n_expert"], c["d"], c["ff"], tg, gate, tu, up, td, down)
        else:
            from . import ep
            d, ff = c["d"], c["ff"]
            ctx.upload_experts(l, c["n_expert"], d, ff, tg, ep.slice_experts(tg, gate, ff, d, block), tu,
                               ep.slice_experts(tu, up, ff, d, block), td, ep.slice_experts(td, down, d, ff, block),
                               first_expert=block.first, n_local=block.count)
        ctx.upload_router(l, by[(l, "ffn_gate_inp")][1], c["k"], c["norm_topk"], c["weights_scale"])
