"""Helpers shared by the GPU tests: seeded MoE layers and device copies."""
import numpy as np

from kestrel_b200 import ggml as G


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def tol_ok(got, ref, tol=1e-3):
    """The reference's criterion (crates/kestrel-engine/tests/oracle.rs:75-78):
    max|got - ref| <= tol * max(max|ref|, 1)."""
    scale = max(float(np.abs(ref).max(initial=0.0)), 1.0)
    err = float(np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64)).max(initial=0.0))
    return err <= tol * scale, err, scale


def make_layer(E, k, d, ff, t_gate=G.Q4_K, t_down=G.Q6_K, seed=0, router_bias=None):
    """A seeded MoE layer: weights N(0, 0.02) quantised with this project's
    quantizer, F32 router N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    gate = G.quantize(t_gate, rng.standard_normal((E * ff, d), dtype=np.float32) * np.float32(0.02))
    up = G.quantize(t_gate, rng.standard_normal((E * ff, d), dtype=np.float32) * np.float32(0.02))
    down = G.quantize(t_down, rng.standard_normal((E * d, ff), dtype=np.float32) * np.float32(0.02))
    router = (rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    return dict(E=E, k=k, d=d, ff=ff, t_gate=t_gate, t_down=t_down, gate=gate, up=up, down=down, router=router)


def upload(ctx, layer_id, L, norm_topk=True, weights_scale=0.0):
    ctx.upload_experts(layer_id, L["E"], L["d"], L["ff"], L["t_gate"], L["gate"], L["t_gate"], L["up"],
                       L["t_down"], L["down"])
    ctx.upload_router(layer_id, L["router"], L["k"], norm_topk, weights_scale)


def oracle_layer(oracle, L, h, norm_topk=True, weights_scale=0.0):
    return oracle.moe_ffn(h, L["router"], L["k"], L["t_gate"], L["gate"], L["t_gate"], L["up"], L["t_down"],
                          L["down"], L["ff"], norm_topk=norm_topk, weights_scale=weights_scale)
