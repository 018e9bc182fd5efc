"""Host-side set-up of expert parallelism: one process per GPU.

Every rank holds a contiguous block of each layer's experts, a full copy of
the router, and its own tokens; `kc_moe_ffn_dev` then exchanges token rows and
result rows with NCCL (see csrc/ep.cu). This module does what the host must do
around that: agree on the NCCL unique id through an existing
torch.distributed group (any backend, gloo included, so the rendezvous also
works on CPU-only hosts), compute each rank's expert block, and slice a
layer's stacked GGUF expert tensors down to that block.

The reference has one process and no expert parallelism; this mirrors its
expert table layout (stacked tensors, expert e at e * slice_bytes,
crates/kestrel-gguf/src/lib.rs:183-189) so that a rank's block is a byte
range of each stacked tensor.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import ggml as G


@dataclass(frozen=True)
class ExpertBlock:
    """Experts [first, first + count) of n_expert, held by one rank."""
    first: int
    count: int
    n_expert: int

    def owner_of(self, e: int) -> int:
        return e // self.count


def expert_block(n_expert: int, world: int, rank: int) -> ExpertBlock:
    """Contiguous block of experts owned by `rank` (world must divide n_expert)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if n_expert % world:
        raise ValueError(f"{n_expert} experts do not split evenly over {world} ranks")
    per = n_expert // world
    return ExpertBlock(first=rank * per, count=per, n_expert=n_expert)


def slice_experts(t: int, stacked: np.ndarray, rows: int, cols: int, block: ExpertBlock) -> np.ndarray:
    """Bytes of experts block.first .. block.first+count-1 of a stacked GGUF
    tensor holding n_expert matrices [rows, cols] of ggml type t."""
    per = rows * G.bytes_for(t, cols)
    flat = np.ascontiguousarray(stacked).reshape(-1).view(np.uint8)
    if flat.size < block.n_expert * per:
        raise ValueError(f"stacked tensor holds {flat.size} bytes, {block.n_expert * per} needed")
    return flat[block.first * per:(block.first + block.count) * per]


def share_unique_id(rank: int, make_id, group=None) -> bytes:
    """Rank 0 calls make_id() (e.g. kestrel_b200.cuda.ep_unique_id) and every
    rank of the torch.distributed group receives the same 128 bytes."""
    import torch.distributed as dist
    obj = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0, group=group)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("expert-parallel unique id must be 128 bytes")
    return bytes(uid)


def join(ctx, rank: int, world: int, group=None) -> None:
    """Join the expert-parallel group of `world` ranks with context `ctx`
    (a kestrel_b200.cuda.Context on this rank's GPU)."""
    from . import cuda
    uid = share_unique_id(rank, cuda.ep_unique_id, group)
    ctx.ep_init(rank, world, uid)
