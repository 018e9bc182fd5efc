"""Small profiling driver: a few MoE layer calls on one GPU with one layer of
weights on the device, for ncu captures. Shapes: c1 = configs[1] (d 2048, 128
experts top-8, ff 768; ~0.4 GB), c2 = configs[2] (d 4096, 8 experts top-2,
ff 14336; ~0.9 GB), c4 = configs[4] shape (d 4096, 128 experts top-8, ff 1536;
~1.6 GB, unskewed routing).

  python -m kestrel_b200.profile_layer --batch 16 --calls 3
  python -m kestrel_b200.profile_layer --config c2 --batch 2048 --calls 2
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
    ap.add_argument("--config", choices=["c1", "c2", "c4"], default="c1")
    args = ap.parse_args()
    E, k, d, ff = {"c1": (128, 8, 2048, 768), "c2": (8, 2, 4096, 14336), "c4": (128, 8, 4096, 1536)}[args.config]
    ctx = Context(0)
    # One stream for torch's tensor work and the library's kernels.
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
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
