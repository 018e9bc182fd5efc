"""Host restatement of the expert-parallel exchange of csrc/ep.cu (test
helper): the home plan of ep_plan_kernel, the owner's local ids
(ep_local_ids_kernel), its return positions (ep_ret_plan_kernel) and the
home combine (combine_kernel over ret_pos), with the experts computed by the
oracle. Used by tests/test_ep_model.py under gloo ranks on CPU.

Layout rules (ep.h): rank r owns experts [r * epr, (r + 1) * epr). The home
sends each token once to every rank owning one of its experts, tokens
ascending per destination. An owner receives the rows of every source in
rank order; the result rows it returns to a source are that source's rows in
received order, each row's local experts ascending. The home combines a
token's result rows in ascending expert id (mul, then add, from +0.0)."""
import numpy as np


def home_plan(ids, world, epr):
    """ep_plan_kernel: send lists, counts and the position of every (token,
    selection) in the concatenated return buffer (owner sections in rank
    order, tokens ascending within a section, a token's experts owned by
    that rank ascending)."""
    n, k = ids.shape
    send = [[s for s in range(n) if any(ids[s, j] // epr == r for j in range(k))] for r in range(world)]
    expect = [sum(1 for s in range(n) for j in range(k) if ids[s, j] // epr == r) for r in range(world)]
    off = np.concatenate([[0], np.cumsum(expect)]).astype(np.int64)
    ret_pos = np.zeros((n, k), np.int64)
    base = [0] * world
    for s in range(n):
        for j in range(k):
            e = int(ids[s, j])
            r = e // epr
            rank = sum(1 for j2 in range(k) if ids[s, j2] // epr == r and ids[s, j2] < e)
            ret_pos[s, j] = off[r] + base[r] + rank
        for r in range(world):
            base[r] += sum(1 for j in range(k) if ids[s, j] // epr == r)
    return send, expect, ret_pos


def owner_compute(recv_rows, recv_ids, first, epr, expert_fn):
    """Owner side: local ids (-1 for other owners' experts), the local
    experts on their rows in received order, and the result rows by
    (received row, selection) position: rows in received order, each row's
    local experts ascending (ep_ret_plan_kernel)."""
    n, k = recv_ids.shape
    loc = np.where((recv_ids >= first) & (recv_ids < first + epr), recv_ids - first, -1)
    y = {}
    for le in range(epr):
        rows = [i for i in range(n) for j in range(k) if loc[i, j] == le]
        if rows:
            y[le] = dict(zip(rows, expert_fn(first + le, recv_rows[rows])))
    pos = np.full((n, k), -1, np.int64)
    out = []
    p = 0
    for i in range(n):
        order = sorted(j for j in range(k) if loc[i, j] >= 0)
        order.sort(key=lambda j: loc[i, j])
        for j in order:
            pos[i, j] = p
            out.append(y[int(loc[i, j])][i])
            p += 1
    return pos, (np.stack(out) if out else np.zeros((0, recv_rows.shape[1]), np.float32))


def combine(ids, w, ret_pos, retrecv):
    """combine_kernel: out[s] = sum over the token's selections in ascending
    expert id of w * y, each step a float32 multiply then add, from +0.0."""
    n, k = ids.shape
    d = retrecv.shape[1]
    out = np.zeros((n, d), np.float32)
    for s in range(n):
        acc = np.zeros(d, np.float32)
        for j in sorted(range(k), key=lambda j: ids[s, j]):
            acc = (acc + (np.float32(w[s, j]) * retrecv[ret_pos[s, j]]).astype(np.float32)).astype(np.float32)
        out[s] = acc
    return out
