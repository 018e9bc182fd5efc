"""One rank of the expert-parallel check (launched by tests/test_gpu_ep.py
through torch.distributed.run, one process per GPU).

Every rank builds the same seeded layer, uploads its contiguous block of
experts and the full router, joins the NCCL group, and runs kc_moe_ffn on its
own tokens. A second, single-GPU context on the same device holding all the
experts runs the union of every rank's tokens (rank-major, the order the
expert-parallel combine reproduces). Each rank routes its own tokens, and the
reference's router product orders its sums by batch size (quant::matmul:
dot for n < 4, gemm_f32 otherwise), so every case keeps each rank's count on
the same side of 4 as the union's. Top-k ids and weights must be identical;
layer outputs must be bit-identical when every expert gets at most 3 rows (the
int8 path, exact on any grouping) and within the reference's tolerance
otherwise (the tensor-core path splits K depending on the batch).
"""
import json
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

import oracle  # noqa: E402
from gpu_util import bits, make_layer, oracle_layer, tol_ok  # noqa: E402
from kestrel_b200 import ep  # noqa: E402
from kestrel_b200.cuda import Context, KestrelCudaError  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    torch.cuda.set_device(rank)
    E, k, d, ff = 16, 4, 512, 768
    L = make_layer(E, k, d, ff, seed=11)
    blk = ep.expert_block(E, world, rank)
    ctx = Context(rank)
    ep.join(ctx, rank, world)
    sl = lambda t, a, rows, cols: ep.slice_experts(t, a, rows, cols, blk)
    ctx.upload_experts(0, E, d, ff, L["t_gate"], sl(L["t_gate"], L["gate"], ff, d), L["t_gate"],
                       sl(L["t_gate"], L["up"], ff, d), L["t_down"], sl(L["t_down"], L["down"], d, ff),
                       first_expert=blk.first, n_local=blk.count)
    ctx.upload_router(0, L["router"], k)
    # Calls of up to 32 tokens per rank exchange through peer memory, larger
    # ones through NCCL. The path is chosen per call from the rank's own token
    # count, so in every case all ranks are on the same side of 32.
    ctx.ep_reserve(32)
    ref = Context(rank)
    ref.upload_experts(0, E, d, ff, L["t_gate"], L["gate"], L["t_gate"], L["up"], L["t_down"], L["down"])
    ref.upload_router(0, L["router"], k)

    results = []
    cases = [[1] * world, [3] + [0] * (world - 1), [16] * world, [40 + 3 * r for r in range(world)], [1] * world,
             [32] * world, [4, 28] + [5] * (world - 2), [32 - 3 * r for r in range(world)]]
    for ci, ns in enumerate(cases):
        rng = np.random.default_rng(100 + ci)
        h_all = rng.standard_normal((sum(ns), d)).astype(np.float32)
        lo = sum(ns[:rank])
        mine = h_all[lo:lo + ns[rank]]
        out, ids, w = ctx.moe_ffn(0, mine)
        # Routing depends on the batch size (quant::matmul's n < 4 dispatch
        # orders the router's sums differently), so ids / weights are compared
        # bit for bit with one GPU routing this rank's own tokens...
        _, own_ids, own_w = ref.moe_ffn(0, mine)
        # ... and the layer output with one GPU running the union of all
        # ranks' tokens, which is also bit-exact when the rank's batch and the
        # union are on the same side of n < 4 and no expert gets 4 rows.
        u_out, all_ids, u_w = ref.moe_ffn(0, h_all)
        r_out, r_ids = u_out[lo:lo + ns[rank]], all_ids[lo:lo + ns[rank]]
        max_rows = int(np.bincount(all_ids.reshape(-1), minlength=E).max()) if all_ids.size else 0
        same_side = (ns[rank] < 4) == (sum(ns) < 4)
        res = dict(case=ci, ns=ns, rank=rank, ids=bool(np.array_equal(ids, own_ids)),
                   w=bool(np.array_equal(bits(w), bits(own_w))), max_rows=max_rows, same_side=same_side)
        if same_side and max_rows <= 3:
            res["out_bit_exact"] = bool(np.array_equal(ids, r_ids) and np.array_equal(bits(out), bits(r_out)))
            res["ok"] = res["ids"] and res["w"] and res["out_bit_exact"]
        else:
            ok, err, scale = tol_ok(out, r_out)
            res.update(out_tol=ok, err=err, scale=scale)
            res["ok"] = res["ids"] and res["w"] and ok
        # ... and against the CPU oracle on the union (the reference's own
        # arithmetic): ids where the routing order agrees, the output within
        # the reference's tolerance.
        o_out, o_ids, _ = oracle_layer(oracle, L, h_all)
        ok_o, err_o, scale_o = tol_ok(out, o_out[lo:lo + ns[rank]])
        res.update(oracle_tol=ok_o, oracle_err=err_o)
        res["ok"] = res["ok"] and ok_o
        results.append(res)
    # A call whose ranks take different exchange paths (rank 0 above the
    # reserved capacity, the others within it) must fail on every rank with
    # KC_ERR_STATE, quickly, and the next call on one path must work again.
    rng = np.random.default_rng(99)
    n_mixed = 40 if rank == 0 else 2
    try:
        ctx.moe_ffn(0, rng.standard_normal((n_mixed, d)).astype(np.float32))
        mixed = "no error"
    except KestrelCudaError as e:
        mixed = "state" if e.code == 7 else f"code {e.code}: {e}"
    # The next call (2 tokens per rank, all on the peer path): ids as one GPU
    # routes this rank's own tokens, the output within the tolerance of one
    # GPU running the union (a union of 4 or more tokens routes in gemm order).
    h_after = np.random.default_rng(100).standard_normal((2 * world, d)).astype(np.float32)
    out_a, ids_a, _ = ctx.moe_ffn(0, h_after[2 * rank:2 * rank + 2])
    _, own_ids_a, _ = ref.moe_ffn(0, h_after[2 * rank:2 * rank + 2])
    u_a, _, _ = ref.moe_ffn(0, h_after)
    ids_ok = bool(np.array_equal(ids_a, own_ids_a))
    tol_a, err_a, _ = tol_ok(out_a, u_a[2 * rank:2 * rank + 2])
    after_ok = ids_ok and tol_a
    results.append(dict(case="mixed-path", rank=rank, mixed=mixed, after_ok=after_ok, after_ids=ids_ok,
                        after_err=err_a, ok=mixed == "state" and after_ok))
    gathered = [None] * world
    dist.all_gather_object(gathered, results)
    ctx.close()
    ref.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        flat = [r for rs in gathered for r in rs]
        print(json.dumps(flat))
        sys.exit(0 if all(r["ok"] for r in flat) else 1)


if __name__ == "__main__":
    main()
