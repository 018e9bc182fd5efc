"""Small profiling driver: a few MoE layer calls at configs[1] shape on one
GPU (one layer of weights, ~0.4 GB on the device), for ncu captures.

  python -m kestrel_b200.profile_layer --batch 16 --calls 3
"""
from __future__ import annotations

import argparse

import torch

from . import ggml as G
from .cuda import Context


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--layers", type=int, default=1)
    args = ap.parse_args()
    E, k, d, ff = 128, 8, 2048, 768
    ctx = Context(0)
    g = torch.Generator(device="cuda").manual_seed(0)
    for layer in range(args.layers):
        mats = {}
        for name, t, rows, cols in (("gate", G.Q4_K, E * ff, d), ("up", G.Q4_K, E * ff, d),
                                    ("down", G.Q6_K, E * d, ff)):
            x = torch.randn((rows, cols), generator=g, device="cuda") * 0.02
            out = torch.empty((rows, G.bytes_for(t, cols)), dtype=torch.uint8, device="cuda")
            ctx.quantize_dev(t, x, out)
            mats[name] = out
            del x
        router = torch.randn((E, d), generator=g, device="cuda") * 0.02
        ctx.upload_experts(layer, E, d, ff, G.Q4_K, mats["gate"], G.Q4_K, mats["up"], G.Q6_K, mats["down"])
        ctx.upload_router(layer, router, k)
        del mats
    torch.cuda.empty_cache()
    h = torch.randn((args.batch, d), generator=g, device="cuda")
    out = torch.empty_like(h)
    ctx.reserve(args.batch)
    for i in range(args.calls):
        ctx.moe_ffn_dev(i % args.layers, h, out)
    ctx.sync()
    torch.cuda.synchronize()
    print("ok", float(out.abs().sum()))
    ctx.close()


if __name__ == "__main__":
    main()
