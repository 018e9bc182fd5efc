"""The algorithmic bytes behind bench.py's roofline line: bytes per expert
from the block formats (Q4_K 144 B and Q6_K 210 B per 256 weights,
GgmlType::bytes_for, crates/kestrel-gguf/src/types.rs:185-191), counted once per distinct
routed expert of a call, plus the router matrix and the activations in and
out; the split between the int8 path (1-3 rows) and the n >= 4 path follows
quant::matmul's dispatch (quant.rs:229-339)."""
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402
from kestrel_b200 import ggml as G  # noqa: E402


@pytest.fixture(params=sorted(bench.CONFIGS))
def cfg(request, monkeypatch):
    c = dict(bench.CONFIGS[request.param])
    monkeypatch.setattr(bench, "CFG", c)
    return c


def expert_bytes_from_formats(c):
    """Gate and up [ff, d] Q4_K, down [d, ff] Q6_K, from the block table."""
    return 2 * c["ff"] * G.bytes_for(G.Q4_K, c["d"]) + c["d"] * G.bytes_for(G.Q6_K, c["ff"])


def test_bytes_per_expert_matches_block_formats(cfg):
    assert bench.bytes_per_expert() == expert_bytes_from_formats(cfg)
    assert bench.router_bytes() == cfg["E"] * cfg["d"] * 4


def test_headline_figures():
    c = bench.CONFIGS["c1"]
    assert expert_bytes_from_formats(c) == 3_059_712
    assert 2 * c["ff"] * G.bytes_for(G.Q4_K, c["d"]) == 1_769_472
    assert c["d"] * G.bytes_for(G.Q6_K, c["ff"]) == 1_290_240


def test_distinct_experts_counted_once_and_split_by_rows(cfg):
    E, k, B = cfg["E"], cfg["k"], 16
    # Experts 0..4 get 1, 2, 3, 4 and B rows where a token can hold all five
    # (k >= 5); every token's remaining picks go to experts 5, 6, ... in turn.
    want = [1, 2, 3, 4, B] if k >= 5 else None
    ids = np.zeros((B, k), dtype=np.int32)
    nxt = 5
    for t in range(B):
        picks = [e for e, n in enumerate(want) if t < n] if want else []
        while len(picks) < k:
            if nxt % E not in picks:
                picks.append(nxt % E)
            nxt += 1
        ids[t] = picks
    cnt = np.bincount(ids.reshape(-1), minlength=E)
    if want:
        assert list(cnt[:5]) == want
    small = int(((cnt >= 1) & (cnt <= 3)).sum())
    large = int((cnt >= 4).sum())
    got = bench.algorithmic_bytes(ids, B)
    gate_up = 2 * cfg["ff"] * G.bytes_for(G.Q4_K, cfg["d"])
    down = cfg["d"] * G.bytes_for(G.Q6_K, cfg["ff"])
    assert got["experts"] == small + large == int((cnt > 0).sum())
    assert got["total"] == (small + large) * (gate_up + down) + E * cfg["d"] * 4 + B * cfg["d"] * 8
    assert got["gate_up_int8"] == small * gate_up and got["down_int8"] == small * down
    assert got["gate_up_f32"] == large * gate_up and got["down_f32"] == large * down


def test_expert_block_counts_only_its_experts(monkeypatch):
    monkeypatch.setattr(bench, "CFG", dict(bench.CONFIGS["c1"]))
    E, k, B = 128, 8, 16
    rng = np.random.default_rng(3)
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(B)]).astype(np.int32)
    whole = bench.algorithmic_bytes(ids, B)
    parts = [bench.algorithmic_bytes(ids, B, SimpleNamespace(first=f, count=32)) for f in range(0, E, 32)]
    assert sum(p["experts"] for p in parts) == whole["experts"]
    fixed = bench.router_bytes() + B * 2048 * 8
    assert sum(p["total"] - fixed for p in parts) == whole["total"] - fixed
