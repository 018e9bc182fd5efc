"""Layer calls with host-streamed experts (kc_upload_experts_streamed), one GPU.

  python -m kestrel_b200.stream_bench --slots 2048 --batch 1
  python -m kestrel_b200.stream_bench --slots 2048 --batch 16 --prefetch

configs[1]'s MoE layer (Qwen3-30B-A3B: d_model 2048, 128 experts top-8 of
width 768, Q4_K gate/up and Q6_K down) over 48 layers whose experts stay in
pinned host memory (18.8 GB); `--slots` HBM cache slots (+ `--scratch`,
`--spec`; `--policy lfru|lru`) hold the resident ones. Each call is one layer
(cycling through the 48) on B tokens of N(0, 1) input, so routing is close to
uniform and the hit rate is about slots / 6144 once the cache is warm.

With --prefetch every call first announces the NEXT call's experts through
kc_expert_prefetch (the ids of the next call's tokens, routed beforehand with
kc_router_logits_dev + kc_route_dev: an exact prediction, an upper bound on what router lookahead
can do), so their copies overlap the current call.

Prints one JSON line: calls/s and tokens/s over the timed calls (CUDA events
on the library's stream; every call synchronises once on its routed ids), the
cache counters of the timed calls, the host->HBM bytes they copied and their
GB/s, and a plain pinned host->device copy rate measured in the same process
(the bound on copied bytes). The same calls on resident layers are timed for
comparison when --resident is given.
"""
from __future__ import annotations

import argparse
import json

import numpy as np

from . import ggml as G

D, E, K, FF, N_LAYERS = 2048, 128, 8, 768, 48


def make_layers(ctx, torch, streamed: bool, seed: int = 0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    bufs = {n: torch.empty((rows, G.bytes_for(t, cols)), dtype=torch.uint8, device="cuda")
            for n, t, rows, cols in (("gate", G.Q4_K, E * FF, D), ("up", G.Q4_K, E * FF, D), ("down", G.Q6_K, E * D, FF))}
    x = torch.empty((E * FF, D), dtype=torch.float32, device="cuda")
    routers = []
    for layer in range(N_LAYERS):
        for n, t in (("gate", G.Q4_K), ("up", G.Q4_K), ("down", G.Q6_K)):
            xv = x.view(E * D, FF) if n == "down" else x
            xv.normal_(0.0, 0.02, generator=g)
            ctx.quantize_dev(t, xv, bufs[n])
        router = torch.empty((E, D), dtype=torch.float32, device="cuda").normal_(0.0, 0.02, generator=g)
        up = ctx.upload_experts_streamed if streamed else ctx.upload_experts
        up(layer, E, D, FF, G.Q4_K, bufs["gate"], G.Q4_K, bufs["up"], G.Q6_K, bufs["down"])
        ctx.upload_router(layer, router, K)
        routers.append(router)
    del x, bufs
    torch.cuda.empty_cache()
    return routers


def pinned_h2d_gbs(torch, nbytes=1 << 30, reps=5) -> float:
    src = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dst.copy_(src, non_blocking=True)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        dst.copy_(src, non_blocking=True)
    b.record()
    b.synchronize()
    return reps * nbytes / (a.elapsed_time(b) / 1e3) / 1e9


def run_calls(ctx, torch, hs, outs, calls, routers=None, ids_next=None):
    """Device time (s) of `calls` layer calls; with routers, each call first
    prefetches the next call's experts."""
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record(stream)
    for i in range(calls):
        if routers is not None:
            j = i + 1
            ctx.router_logits_dev(routers[j % N_LAYERS], hs[j % len(hs)], ids_next[2])
            ctx.route_dev(ids_next[2], K, ids_next[0], ids_next[1])
            nxt = np.unique(ids_next[0].cpu().numpy())
            ctx.expert_prefetch(j % N_LAYERS, nxt)
        ctx.moe_ffn_dev(i % N_LAYERS, hs[i % len(hs)], outs[i % len(outs)], n_tok=hs[0].shape[0])
    b.record(stream)
    b.synchronize()
    return a.elapsed_time(b) / 1e3


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--slots", type=int, default=2048)
    ap.add_argument("--scratch", type=int, default=64)
    ap.add_argument("--spec", type=int, default=64)
    ap.add_argument("--policy", choices=["lfru", "lru"], default="lfru")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--calls", type=int, default=480)
    ap.add_argument("--warmup", type=int, default=960, help="untimed calls that warm the cache first")
    ap.add_argument("--prefetch", action="store_true")
    ap.add_argument("--resident", action="store_true", help="also time the same calls on resident layers")
    args = ap.parse_args()
    import torch
    from .cuda import EXPERT_POLICY_LFRU, EXPERT_POLICY_LRU, Context
    torch.cuda.set_device(0)
    ctx = Context(0)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    B = args.batch
    gen = torch.Generator(device="cuda").manual_seed(5)
    hs = [torch.randn((B, D), generator=gen, device="cuda") for _ in range(97)]
    outs = [torch.empty((B, D), device="cuda") for _ in range(2)]
    ids_next = (torch.empty((B, K), dtype=torch.int32, device="cuda"), torch.empty((B, K), device="cuda"),
                torch.empty((B, E), device="cuda"))
    routers = make_layers(ctx, torch, streamed=True)
    ctx.expert_cache_reserve(args.slots, args.scratch,
                             EXPERT_POLICY_LRU if args.policy == "lru" else EXPERT_POLICY_LFRU, spec=args.spec)
    pf = routers if args.prefetch else None
    run_calls(ctx, torch, hs, outs, args.warmup, pf, ids_next)
    s0 = ctx.expert_cache_stats()
    t = run_calls(ctx, torch, hs, outs, args.calls, pf, ids_next)
    s1 = ctx.expert_cache_stats()
    dx = {k: s1[k] - s0[k] for k in s1 if k not in ("capacity", "scratch", "spec", "cached")}
    line = {
        "metric": "streamed_moe_layer_tokens_per_s", "value": args.calls * B / t, "unit": "tokens/s",
        "calls_per_s": args.calls / t, "ms_per_call": 1e3 * t / args.calls, "batch": B,
        "workload": "configs[1] MoE layer, 48 layers of experts in pinned host memory (18.8 GB)",
        "slots": args.slots, "scratch": args.scratch, "spec": args.spec, "policy": args.policy,
        "prefetch_next_call": bool(args.prefetch), "cached_after": s1["cached"],
        "counters": dx, "hit_rate": dx["hits"] / max(1, dx["requests"]),
        "h2d_bytes_per_call": dx["bytes_read"] / args.calls, "h2d_gbs": dx["bytes_read"] / t / 1e9,
        "h2d_copy_peak_gbs": pinned_h2d_gbs(torch),
        "timing": "CUDA events on the library's stream around the timed calls, after the warm-up calls",
    }
    line["h2d_frac"] = line["h2d_gbs"] / line["h2d_copy_peak_gbs"]
    if args.resident:
        ctx.close()
        torch.cuda.empty_cache()
        ctx = Context(0)
        ctx.set_stream(torch.cuda.current_stream().cuda_stream)
        make_layers(ctx, torch, streamed=False)
        run_calls(ctx, torch, hs, outs, 96)
        tr = run_calls(ctx, torch, hs, outs, args.calls)
        line["resident_ms_per_call"] = 1e3 * tr / args.calls
    print(json.dumps(line))
    ctx.close()


if __name__ == "__main__":
    main()
