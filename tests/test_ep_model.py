"""The expert-parallel exchange restated on the host (tests/ep_model.py) and
run across gloo ranks on CPU (world size 2 and 4): each rank routes its own
tokens, sends rows to the experts' owners, owners run their experts with the
oracle, result rows go back, and each home combines in ascending expert id.
Every rank's output must equal the oracle's moe_ffn over the union of all
ranks' tokens bit for bit -- the per-expert batches are the union's (sources
in rank order, tokens ascending), so this holds on the int8 and the f32
path alike. The router's sums follow quant::matmul's dispatch (quant.rs:241:
dot for n < 4; gemm_f32 otherwise, whose tokens outside whole 4-token blocks
take dot_f32's order), so every case either keeps all batches below 4 tokens
or makes every rank's count, and so every rank's offset in the union, a
multiple of 4: each token then gets the same summation order alone as in the
union."""
import os
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

CASES = {2: [[1, 1], [3, 0], [16, 16], [4, 8], [8, 4]],
         4: [[1, 1, 1, 0], [4, 4, 8, 4], [1, 0, 1, 1], [12, 4, 8, 0]]}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    sys.path[:0] = [ROOT, HERE]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle
    from kestrel_b200 import ggml as G
    from gpu_util import make_layer
    import ep_model as M

    E, k, d, ff = 16, 4, 256, 256
    L = make_layer(E, k, d, ff, seed=7)
    epr = E // world
    rbg, rbd = G.bytes_for(G.Q4_K, d), G.bytes_for(G.Q6_K, ff)

    def expert_fn(e, xs):
        return oracle.expert_ffn(G.Q4_K, L["gate"].reshape(-1)[e * ff * rbg:(e + 1) * ff * rbg],
                                 G.Q4_K, L["up"].reshape(-1)[e * ff * rbg:(e + 1) * ff * rbg],
                                 G.Q6_K, L["down"].reshape(-1)[e * d * rbd:(e + 1) * d * rbd], d, ff, xs)

    results = []
    for ci, ns in enumerate(CASES[world]):
        h_all = np.random.default_rng(500 + ci).standard_normal((sum(ns), d)).astype(np.float32)
        lo = sum(ns[:rank])
        mine = h_all[lo:lo + ns[rank]]
        if ns[rank]:
            logits = oracle.matmul(0, L["router"].view(np.uint8), E, d, mine)
            ids, w = oracle.route(logits, k)
        else:
            ids, w = np.zeros((0, k), np.int32), np.zeros((0, k), np.float32)
        send, expect, ret_pos = M.home_plan(ids.astype(np.int64), world, epr)
        # rows (and their k ids / weights) to every owner
        out_msgs = [(mine[send[r]], ids[send[r]], w[send[r]]) for r in range(world)]
        gathered = [None] * world
        dist.all_gather_object(gathered, out_msgs)
        recv = [gathered[src][rank] for src in range(world)]  # sources in rank order
        counts = [len(x[0]) for x in recv]
        rows = np.concatenate([x[0] for x in recv]) if sum(counts) else np.zeros((0, d), np.float32)
        rids = np.concatenate([x[1] for x in recv]).astype(np.int64) if sum(counts) else np.zeros((0, k), np.int64)
        pos, yret = M.owner_compute(rows, rids, rank * epr, epr, expert_fn)
        # result rows back: source q's rows are contiguous in received order
        starts = np.concatenate([[0], np.cumsum(counts)])
        sections = []
        for src in range(world):
            p = pos[starts[src]:starts[src + 1]]
            p = p[p >= 0]
            sections.append(yret[p.min():p.max() + 1] if p.size else np.zeros((0, d), np.float32))
        back = [None] * world
        dist.all_gather_object(back, sections)
        retrecv = np.concatenate([back[r][rank] for r in range(world)]) if ns[rank] else np.zeros((0, d), np.float32)
        assert len(retrecv) == sum(expect)
        out = M.combine(ids.astype(np.int64), w, ret_pos, retrecv) if ns[rank] else np.zeros((0, d), np.float32)
        u_out, u_ids, u_w = oracle.moe_ffn(h_all, L["router"], k, G.Q4_K, L["gate"], G.Q4_K, L["up"], G.Q6_K,
                                           L["down"], ff)
        ok = (np.array_equal(ids, u_ids[lo:lo + ns[rank]]) and
              np.array_equal(out.view(np.uint32), u_out[lo:lo + ns[rank]].view(np.uint32)))
        results.append((ci, ok))
    q.put((rank, results))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_exchange_model_matches_union_oracle(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    bad = [(r, ci) for r, res in got for ci, ok in res if not ok]
    assert not bad, bad


def test_home_plan_positions_are_a_permutation():
    """Return positions cover the return buffer exactly once; within an owner's
    section a token's experts are ascending."""
    sys.path[:0] = [HERE]
    import ep_model as M
    rng = np.random.default_rng(3)
    for world, E, k, n in ((2, 8, 2, 5), (4, 16, 4, 9), (8, 128, 8, 16)):
        ids = np.stack([rng.choice(E, size=k, replace=False) for _ in range(n)])
        send, expect, ret_pos = M.home_plan(ids, world, E // world)
        assert sorted(ret_pos.reshape(-1).tolist()) == list(range(n * k))
        assert sum(expect) == n * k
        for s in range(n):
            for r in range(world):
                js = [j for j in range(k) if ids[s, j] // (E // world) == r]
                assert [ids[s, j] for j in sorted(js, key=lambda j: ret_pos[s, j])] == sorted(ids[s, js].tolist())
