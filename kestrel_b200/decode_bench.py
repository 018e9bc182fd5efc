"""Whole-model greedy decode throughput (kc_model_*), one GPU.

  python -m kestrel_b200.decode_bench --model c0 --prompt 64 --gen 64
  python -m kestrel_b200.decode_bench --model c3 --prompt 512 --gen 256
  python -m kestrel_b200.decode_bench --model c3 --batch 8   # 8 sequences in lockstep
  python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \
      -m kestrel_b200.decode_bench --model c3     # expert parallel over N GPUs

With N ranks (one process per GPU) every MoE layer's experts are sharded in
contiguous blocks (rank r holds E/N of them, the dense weights are
replicated), and every rank decodes its own sequence: each step, every rank's
token goes through its layers, exchanging rows and results with the experts'
owners over NVLink peer memory inside each layer call. The reported value is
the tokens all ranks decode per second (weak scaling: one sequence per GPU),
timed with CUDA events on each rank, max over ranks.

c0 is configs[0] (kestrel_b200.synth.CONFIG0, weights made on the host). c3
is configs[3]: a random-init Qwen3-30B-A3B-architecture model -- 48 layers,
d_model 2048, 32 query / 4 KV heads of 128, vocab 151936, 128 experts top-8
of width 768, Q4_K gate/up and Q6_K down experts, Q4_K attention and
embedding, Q6_K output head, RoPE theta 1e6, n_ctx 4096 -- with its ~20 GB of
weights drawn N(0, 0.02) and quantized on the GPU. Prints one JSON line:
prefill time of the prompt, decode tokens/s of the greedy steps (batch 1),
and the weight bytes one decode step streams.

Timing: the prompt is prefilled by kc_model_forward (CUDA events around it);
the decode steps are then timed alone -- kc_model_generate continues from
the cached prompt with its first token and runs n_gen one-row forwards,
bracketed by CUDA events on the library's stream.

--batch B (B > 1): B independent sequences (prompts of the same length, other
seeds) in lockstep: each prompt is prefilled alone (kc_model_prefill_seq,
all B timed together), then kc_model_decode_seqs runs n_gen + 1 tokens per
sequence -- n_gen steps of B rows, each row computed as a batch of one --
timed alone. The value counts B * n_gen tokens per decode time.

--forced: the decode steps are fed seeded random tokens (one kc_model_forward
of one row each) instead of the greedy token: with random weights greedy
decoding soon repeats one token and routes every step to the same experts,
while forced tokens route like varied text.

--streamed SLOTS: every layer's experts stay in pinned host memory
(kc_upload_experts_streamed) and are copied on demand into SLOTS HBM cache
slots (+ --scratch slots; --policy lfru|lru), with router lookahead unless
--no-lookahead. The line then carries the cache counters of the decode steps
(hits, misses, prefetches, bytes copied), their host->HBM GB/s, and a plain
pinned host->device copy rate measured in the same process for scale.
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


def load_on_gpu(ctx, torch, cfg, n_ctx, seed=0, block=None, streamed=False):
    """Declare cfg and make every weight on the GPU (N(0, 0.02) quantized with
    kc_quantize_dev; norms 1.0). With an expert block (expert parallelism)
    only that block of every layer's experts is uploaded; the weights are
    drawn identically on every rank."""
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
        if streamed:
            ctx.upload_experts_streamed(l, E, d, ff, cfg["t_gate"], gate, cfg["t_gate"], up, cfg["t_down"], down)
        elif block is None:
            ctx.upload_experts(l, E, d, ff, cfg["t_gate"], gate, cfg["t_gate"], up, cfg["t_down"], down)
        else:
            r0, r1 = block.first, block.first + block.count
            ctx.upload_experts(l, E, d, ff, cfg["t_gate"], gate[r0 * ff:r1 * ff], cfg["t_gate"], up[r0 * ff:r1 * ff],
                               cfg["t_down"], down[r0 * d:r1 * d], first_expert=block.first, n_local=block.count)
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


def pinned_h2d_gbs(torch, nbytes=1 << 30, reps=5) -> float:
    """A plain host->device copy from pinned memory (the bound on streamed
    experts), CUDA events, GB/s."""
    src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dst.copy_(src, non_blocking=True)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        dst.copy_(src, non_blocking=True)
    b.record()
    b.synchronize()
    gbs = reps * nbytes / (a.elapsed_time(b) / 1e3) / 1e9
    del src, dst
    return gbs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=["c0", "c3"], default="c0")
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--gen", type=int, default=None)
    ap.add_argument("--n-ctx", type=int, default=None)
    ap.add_argument("--f32-prefill", action="store_true")
    ap.add_argument("--no-warmup", action="store_true", help="skip the warm-up generation (profiling runs)")
    ap.add_argument("--batch", type=int, default=1, help="independent sequences decoded in lockstep")
    ap.add_argument("--ep-tokens", type=int, default=0,
                    help="expert parallelism: tokens per rank and call reserved for the peer-memory exchange "
                         "(default max(8, batch))")
    ap.add_argument("--streamed", type=int, default=0, help="HBM cache slots for host-streamed experts (0: resident)")
    ap.add_argument("--scratch", type=int, default=128)
    ap.add_argument("--policy", choices=["lfru", "lru"], default="lfru")
    ap.add_argument("--no-lookahead", action="store_true")
    ap.add_argument("--forced", action="store_true", help="decode steps on seeded random tokens (teacher forcing)")
    args = ap.parse_args()
    import os

    import torch
    from .cuda import EXPERT_POLICY_LRU, EXPERT_POLICY_LFRU, OPT_F32_PREFILL, OPT_LOOKAHEAD, Context
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    ctx = Context(local)
    # One stream for torch's weight generation and the library's kernels.
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    block = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        from . import ep
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        ep.join(ctx, rank, world)
    if args.model == "c0":
        cfg = dict(synth.CONFIG0)
        n_prompt, n_gen = args.prompt or 64, args.gen or 64
        n_ctx = args.n_ctx or 256
        if world > 1:
            from . import ep
            block = ep.expert_block(cfg["n_expert"], world, rank)
        synth.load_cuda(ctx, synth.make_model(cfg, seed=0), n_ctx, block=block, streamed=args.streamed > 0)
    else:
        cfg = dict(C3)
        n_prompt, n_gen = args.prompt or 512, args.gen or 256
        n_ctx = args.n_ctx or 4096
        if world > 1:
            from . import ep
            block = ep.expert_block(cfg["n_expert"], world, rank)
        load_on_gpu(ctx, torch, cfg, n_ctx, block=block, streamed=args.streamed > 0)
    if args.streamed:
        ctx.expert_cache_reserve(args.streamed, args.scratch,
                                 EXPERT_POLICY_LRU if args.policy == "lru" else EXPERT_POLICY_LFRU)
        ctx.set_option(OPT_LOOKAHEAD, 0 if args.no_lookahead else 1)
    if world > 1:
        # Layer calls of up to --ep-tokens tokens per rank exchange through
        # peer memory (decode steps: one token, or --batch rows), larger ones
        # (prompt chunks of up to 256 tokens) through NCCL. Every owner runs
        # its expert pipeline over the reserved capacity of all sources, so a
        # reservation sized for the prompt chunks slows every decode step.
        ctx.ep_reserve(args.ep_tokens if args.ep_tokens > 0 else max(8, args.batch))
    ctx.set_option(OPT_F32_PREFILL, 1 if args.f32_prefill else 0)
    B = max(1, args.batch)
    prompts = [[int(t) for t in np.random.default_rng(1 + rank * B + s).integers(0, cfg["n_vocab"], n_prompt)]
               for s in range(B)]
    prompt = prompts[0]
    stream = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    finite, absmax = None, None
    if B == 1:
        # Warm-up (workspace sizing, first launches), then timed runs.
        if not args.no_warmup:
            ctx.model_generate(prompt[:8], 4)
            ctx.model_truncate(0)
        torch.cuda.synchronize()
        ev[0].record(stream)
        logits, first = ctx.model_forward(prompt)
        ev[1].record(stream)
        ev[1].synchronize()
        t_prefill = ev[0].elapsed_time(ev[1]) / 1e3
        finite = bool(np.isfinite(logits).all())
        absmax = float(np.abs(logits[np.isfinite(logits)]).max()) if finite or np.isfinite(logits).any() else None
        # Decode alone: continue from the cached prompt with its greedy token;
        # every one of the n_gen forwards is a one-row decode step.
        torch.cuda.synchronize()
        xs0 = ctx.expert_cache_stats()
        forced = [int(t) for t in np.random.default_rng(97).integers(0, cfg["n_vocab"], n_gen)]
        ev[2].record(stream)
        if args.forced:
            toks = [first]
            for t in forced:
                toks.append(ctx.model_forward([t])[1])
        else:
            toks = [first] + list(ctx.model_generate([first], n_gen))
        ev[3].record(stream)
        ev[3].synchronize()
        t_decode = max(1e-9, ev[2].elapsed_time(ev[3]) / 1e3)
    else:
        ctx.model_set_sequences(B)
        if not args.no_warmup:
            for s in range(B):
                ctx.model_prefill_seq(s, prompts[s][:8])
            ctx.model_decode_seqs(B, 4)
        torch.cuda.synchronize()
        ev[0].record(stream)
        firsts = [ctx.model_prefill_seq(s, prompts[s]) for s in range(B)]
        ev[1].record(stream)
        ev[1].synchronize()
        t_prefill = ev[0].elapsed_time(ev[1]) / 1e3
        # n_gen + 1 tokens per sequence: the pending token, then n_gen steps.
        torch.cuda.synchronize()
        xs0 = ctx.expert_cache_stats()
        ev[2].record(stream)
        out = ctx.model_decode_seqs(B, n_gen + 1)
        ev[3].record(stream)
        ev[3].synchronize()
        t_decode = max(1e-9, ev[2].elapsed_time(ev[3]) / 1e3)
        assert [o[0] for o in out] == firsts
        toks = out[0]
    xs1 = ctx.expert_cache_stats()
    if world > 1:
        import torch.distributed as dist
        tt = torch.tensor([t_decode, t_prefill], dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_decode, t_prefill = float(tt[0]), float(tt[1])
    steps = n_gen
    k = cfg["k"]
    # Weight bytes of a step: with B rows, the experts the step's rows choose
    # (counted as B * k distinct, an upper bound: the union is smaller when
    # rows share experts).
    sb = step_bytes(cfg, min(cfg["n_expert"], k * B))
    line = {
        "metric": "decode_tokens_per_s", "value": world * B * steps / t_decode, "unit": "tokens/s", "n_gpus": world,
        "batch": B, "sequences": world * B, "parallelism": f"ep{world}" if world > 1 else "single",
        "scaling": f"weak ({B} sequence(s) per GPU)" if world > 1 else None,
        "model": cfg["name"], "prompt_tokens": n_prompt, "generated": n_gen,
        "ms_per_step": 1e3 * t_decode / steps, "ms_per_token": 1e3 * t_decode / steps / B,
        "prefill_ms": 1e3 * t_prefill, "prefill_tokens_per_s": B * n_prompt / t_prefill,
        "step_weight_bytes": sb, "step_gbs": sb / (t_decode / steps) / 1e9,
        "step_bytes_note": "exact" if B == 1 else "upper bound: B * k experts per layer counted distinct",
        "timing": "CUDA events on the library's stream: the prompts' prefill, then the decode steps alone "
                  + ("(kc_model_generate continuing from the cached prompt)" if B == 1 else
                     "(kc_model_decode_seqs after kc_model_prefill_seq of every sequence)"),
        "f32_prefill": bool(args.f32_prefill), "tokens_head": toks[:8], "forced_tokens": bool(args.forced),
        "prompt_logits_finite": finite, "prompt_logits_absmax": absmax,
    }
    if args.streamed:
        dx = {k: xs1[k] - xs0[k] for k in xs1 if k not in ("capacity", "scratch", "spec", "cached")}
        line["streamed"] = {
            "slots": args.streamed, "scratch": args.scratch, "policy": args.policy,
            "lookahead": not args.no_lookahead, "slot_bytes_note": "one expert's gate + up + down",
            "host_store_bytes": cfg["n_layer"] * cfg["n_expert"] * (
                2 * cfg["ff"] * G.bytes_for(cfg["t_gate"], cfg["d"]) + cfg["d"] * G.bytes_for(cfg["t_down"], cfg["ff"])),
            "decode": dx, "hit_rate": dx["hits"] / max(1, dx["requests"]),
            "lookahead_recall": dx["lookahead_correct"] / max(1, dx["lookahead_predicted"]),
            "h2d_gbs": dx["bytes_read"] / t_decode / 1e9,
            "h2d_copy_peak_gbs": pinned_h2d_gbs(torch),
        }
    if rank == 0:
        print(json.dumps(line))
    ctx.close()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
