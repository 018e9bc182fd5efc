"""Host side of expert parallelism on CPU (gloo, world size 2): the NCCL
unique-id rendezvous through a torch.distributed group, each rank's expert
block, and slicing a stacked GGUF expert tensor to that block."""
import os
import socket
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from kestrel_b200 import ep, ggml as G  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    made = []

    def make():
        made.append(1)
        return bytes(range(128))

    uid = ep.share_unique_id(rank, make)
    blk = ep.expert_block(16, world, rank)
    q.put((rank, uid, len(made), blk.first, blk.count))
    dist.barrier()
    dist.destroy_process_group()


def test_unique_id_rendezvous_and_blocks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(g[1] == bytes(range(128)) for g in got)
    assert [g[2] for g in got] == [1, 0]  # only rank 0 made the id
    assert [(g[3], g[4]) for g in got] == [(0, 8), (8, 8)]


def test_expert_block_rules():
    assert ep.expert_block(128, 8, 3).first == 48
    assert ep.expert_block(128, 8, 3).owner_of(50) == 3
    with pytest.raises(ValueError):
        ep.expert_block(10, 4, 0)
    with pytest.raises(ValueError):
        ep.expert_block(8, 2, 2)


@pytest.mark.parametrize("t", [G.Q4_K, G.Q6_K, G.Q8_0])
def test_slice_experts_is_the_block_of_rows(t):
    E, rows, cols = 4, 3, 256
    rng = np.random.default_rng(0)
    stacked = G.quantize(t, rng.standard_normal((E * rows, cols)).astype(np.float32))
    for r in range(2):
        blk = ep.expert_block(E, 2, r)
        got = ep.slice_experts(t, stacked, rows, cols, blk)
        want = stacked[blk.first * rows:(blk.first + blk.count) * rows].reshape(-1)
        assert np.array_equal(got, want)
