"""Whole-model greedy decode throughput (kc_model_*), one GPU.

  python -m kestrel_b200.decode_bench --model c0 --prompt 64 --gen 64
  python -m kestrel_b200.decode_bench --model c3 --prompt 512 --gen 256

c0 is configs[0] (kestrel_b200.synth.CONFIG0, weights made on the host). c3
is configs[3]: a random-init Qwen3-30B-A3B-architecture model -- 48 layers,
d_model 2048, 32 query / 4 KV heads of 128, vocab 151936, 128 experts top-8
of width 768, Q4_K gate/up and Q6_K down experts, Q4_K attention and
embedding, Q6_K output head, RoPE theta 1e6, n_ctx 4096 -- with its ~20 GB of
weights drawn N(0, 0.02) and quantized on the GPU. Prints one JSON line:
prefill time of the prompt, decode tokens/s of the greedy steps (batch 1),
and the weight bytes one decode step streams.
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np

from . import ggml as G
from . import synth

C3 = dict(name="qwen3-30b-a3b-decode", arch=synth.ARCH_QWEN3, n_layer=48, d=2048, n_head=32, n_kv=4, head_dim=128,
          n_vocab=151936, rope_dim=128, rope_base=1e6, eps=1e-6, n_expert=128, k=8, ff=768, norm_topk=True,
          weights_scale=0.0, t_attn=G.Q4_K, t_embd=G.Q4_K, t_out=G.Q6_K, t_gate=G.Q4_K, t_down=G.Q6_K,
          dense_ff=0)


def load_on_gpu(ctx, torch, cfg, n_ctx, seed=0):
    """Declare cfg and make every weight on the GPU (N(0, 0.02) quantized with
    kc_quantize_dev; norms 1.0)."""
    from .cuda import (T_ATTN_K, T_ATTN_K_NORM, T_ATTN_NORM, T_ATTN_OUT, T_ATTN_Q, T_ATTN_Q_NORM, T_ATTN_V,
                       T_FFN_NORM, T_OUTPUT, T_OUTPUT_NORM, T_TOKEN_EMBD)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    d, nh, nkv, hd = cfg["d"], cfg["n_head"], cfg["n_kv"], cfg["head_dim"]
    ctx.model_init(cfg["n_layer"], d, nh, nkv, hd, cfg["n_vocab"], n_ctx, cfg["rope_dim"], cfg["rope_base"],
                   cfg["eps"], cfg["arch"])

    def quant(t, rows, cols):
        out = torch.empty((rows, G.bytes_for(t, cols)), dtype=torch.uint8, device="cuda")
        step = max(1, (1 << 26) // cols)  # 256 MB of f32 at a time
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            x = torch.randn((r1 - r0, cols), generator=gen, device="cuda") * 0.02
            ctx.quantize_dev(t, x, out[r0:r1])
        return out

    ones = lambda n: torch.ones(n, dtype=torch.float32, device="cuda")
    ctx.model_tensor(-1, T_TOKEN_EMBD, cfg["t_embd"], quant(cfg["t_embd"], cfg["n_vocab"], d), cfg["n_vocab"], d)
    ctx.model_tensor(-1, T_OUTPUT_NORM, G.F32, ones(d), 1, d)
    ctx.model_tensor(-1, T_OUTPUT, cfg["t_out"], quant(cfg["t_out"], cfg["n_vocab"], d), cfg["n_vocab"], d)
    E, ff = cfg["n_expert"], cfg["ff"]
    for l in range(cfg["n_layer"]):
        ctx.model_tensor(l, T_ATTN_NORM, G.F32, ones(d), 1, d)
        ctx.model_tensor(l, T_FFN_NORM, G.F32, ones(d), 1, d)
        if cfg["arch"] == synth.ARCH_QWEN3:
            ctx.model_tensor(l, T_ATTN_Q_NORM, G.F32, ones(hd), 1, hd)
            ctx.model_tensor(l, T_ATTN_K_NORM, G.F32, ones(hd), 1, hd)
        ta = cfg["t_attn"]
        ctx.model_tensor(l, T_ATTN_Q, ta, quant(ta, nh * hd, d), nh * hd, d)
        ctx.model_tensor(l, T_ATTN_K, ta, quant(ta, nkv * hd, d), nkv * hd, d)
        ctx.model_tensor(l, T_ATTN_V, ta, quant(ta, nkv * hd, d), nkv * hd, d)
        ctx.model_tensor(l, T_ATTN_OUT, ta, quant(ta, d, nh * hd), d, nh * hd)
        gate = quant(cfg["t_gate"], E * ff, d)
        up = quant(cfg["t_gate"], E * ff, d)
        down = quant(cfg["t_down"], E * d, ff)
        ctx.upload_experts(l, E, d, ff, cfg["t_gate"], gate, cfg["t_gate"], up, cfg["t_down"], down)
        del gate, up, down
        router = torch.randn((E, d), generator=gen, device="cuda") * 0.02
        ctx.upload_router(l, router, cfg["k"], cfg["norm_topk"], cfg["weights_scale"])
    torch.cuda.synchronize()


def step_bytes(cfg, experts_per_layer) -> int:
    """Weight bytes of one decode step: attention + head + the routed experts."""
    d, nh, nkv, hd = cfg["d"], cfg["n_head"], cfg["n_kv"], cfg["head_dim"]
    attn = (nh * hd + 2 * nkv * hd) * G.bytes_for(cfg["t_attn"], d) + d * G.bytes_for(cfg["t_attn"], nh * hd)
    expert = 2 * cfg["ff"] * G.bytes_for(cfg["t_gate"], d) + d * G.bytes_for(cfg["t_down"], cfg["ff"])
    head = cfg["n_vocab"] * G.bytes_for(cfg["t_out"], d)
    router = cfg["n_expert"] * d * 4
    return cfg["n_layer"] * (attn + router + experts_per_layer * expert) + head


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=["c0", "c3"], default="c0")
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--gen", type=int, default=None)
    ap.add_argument("--n-ctx", type=int, default=None)
    ap.add_argument("--f32-prefill", action="store_true")
    ap.add_argument("--no-warmup", action="store_true", help="skip the warm-up generation (profiling runs)")
    args = ap.parse_args()
    import torch
    from .cuda import OPT_F32_PREFILL, Context
    ctx = Context(0)
    # One stream for torch's weight generation and the library's kernels.
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    if args.model == "c0":
        cfg = dict(synth.CONFIG0)
        n_prompt, n_gen = args.prompt or 64, args.gen or 64
        n_ctx = args.n_ctx or 256
        synth.load_cuda(ctx, synth.make_model(cfg, seed=0), n_ctx)
    else:
        cfg = dict(C3)
        n_prompt, n_gen = args.prompt or 512, args.gen or 256
        n_ctx = args.n_ctx or 4096
        load_on_gpu(ctx, torch, cfg, n_ctx)
    ctx.set_option(OPT_F32_PREFILL, 1 if args.f32_prefill else 0)
    prompt = [int(t) for t in np.random.default_rng(1).integers(0, cfg["n_vocab"], n_prompt)]
    # Warm-up (workspace sizing, first launches), then timed runs.
    if not args.no_warmup:
        ctx.model_generate(prompt[:8], 4)
        ctx.model_truncate(0)
    t0 = time.perf_counter()
    logits, _ = ctx.model_forward(prompt)
    t_prefill = time.perf_counter() - t0
    finite = bool(np.isfinite(logits).all())
    absmax = float(np.abs(logits[np.isfinite(logits)]).max()) if finite or np.isfinite(logits).any() else None
    ctx.model_truncate(0)
    t0 = time.perf_counter()
    toks = ctx.model_generate(prompt, n_gen)
    t_all = time.perf_counter() - t0
    t_decode = max(1e-9, t_all - t_prefill)
    steps = n_gen - 1  # forwards after the prompt
    k = cfg["k"]
    line = {
        "metric": "decode_tokens_per_s", "value": steps / t_decode, "unit": "tokens/s", "n_gpus": 1,
        "batch": 1, "model": cfg["name"], "prompt_tokens": n_prompt, "generated": n_gen,
        "ms_per_token": 1e3 * t_decode / steps, "prefill_ms": 1e3 * t_prefill,
        "prefill_tokens_per_s": n_prompt / t_prefill,
        "step_weight_bytes": step_bytes(cfg, k), "step_gbs": step_bytes(cfg, k) / (t_decode / steps) / 1e9,
        "timing": "wall clock around synchronous kc_model_forward / kc_model_generate calls",
        "f32_prefill": bool(args.f32_prefill), "tokens_head": toks[:8],
        "prompt_logits_finite": finite, "prompt_logits_absmax": absmax,
    }
    print(json.dumps(line))
    ctx.close()


if __name__ == "__main__":
    main()
