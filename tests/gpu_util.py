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


def rel_report(got, ref):
    """Pure elementwise relative error |got - ref| / |ref| over the entries
    whose |ref| is at least 1% of max|ref| (the reference's criterion above
    normalises by the output's scale; this shows the per-element view)."""
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got, np.float64)
    scale = max(float(np.abs(ref).max(initial=0.0)), 1e-30)
    m = np.abs(ref) >= 0.01 * scale
    if not m.any():
        return 0.0, 0.0
    r = np.abs(got[m] - ref[m]) / np.abs(ref[m])
    return float(np.median(r)), float(r.max())


def gpu_layer(ctx, lid, E, k, d, ff, seed, zipf=False):
    """A seeded full-size MoE layer quantised on the GPU with this library's
    quantizer (byte-identical to kestrel_b200.ggml's, which numpy would take
    minutes for at these shapes): Q4_K gate/up + Q6_K down from N(0, 0.02),
    F32 router N(0, 0.02). Uploaded as layer `lid`; returns the host bytes for
    the oracle.

    zipf: configs[4]'s skew. The reference's router has no bias term, so the
    inputs carry it -- feature 0 of every token is 1 (see layer_input) and
    router column 0 holds beta_e = -1.2 * ln(1 + rank(e)) * sigma_logit
    (rank: a seeded permutation), which adds beta_e to expert e's logit and
    makes popularity roughly Zipf s=1.2."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    host = {}
    for name, t, rows, cols in (("gate", G.Q4_K, E * ff, d), ("up", G.Q4_K, E * ff, d), ("down", G.Q6_K, E * d, ff)):
        x = torch.empty((rows, cols), dtype=torch.float32, device="cuda").normal_(0.0, 0.02, generator=g)
        q = torch.empty((rows, G.bytes_for(t, cols)), dtype=torch.uint8, device="cuda")
        ctx.quantize_dev(t, x, q)
        torch.cuda.synchronize()
        host[name] = q.cpu().numpy()
        del x, q
    rng = np.random.default_rng(seed)
    router = (rng.standard_normal((E, d), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    if zipf:
        sigma = 0.02 * np.sqrt(d)  # std of a router logit for N(0, 1) features
        rank = rng.permutation(E)
        router[:, 0] = (-1.2 * np.log1p(rank) * sigma).astype(np.float32)
    host.update(router=router, E=E, k=k, d=d, ff=ff, zipf=zipf)
    ctx.upload_experts(lid, E, d, ff, G.Q4_K, host["gate"], G.Q4_K, host["up"], G.Q6_K, host["down"])
    ctx.upload_router(lid, router, k)
    torch.cuda.empty_cache()
    return host


def layer_input(host, n, seed):
    h = np.random.default_rng(seed).standard_normal((n, host["d"])).astype(np.float32)
    if host["zipf"]:
        h[:, 0] = 1.0
    return h


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


# Oracle tensor kinds (oracle/kestrel_oracle.cpp KO_*) by GGUF name.
ORACLE_KINDS = {"attn_norm": 0, "attn_q": 1, "attn_k": 2, "attn_v": 3, "attn_output": 4, "attn_q_bias": 5,
                "attn_k_bias": 6, "attn_v_bias": 7, "attn_q_norm": 8, "attn_k_norm": 9, "ffn_norm": 10,
                "ffn_gate": 11, "ffn_up": 12, "ffn_down": 13, "ffn_gate_inp": 14, "ffn_gate_exps": 15,
                "ffn_up_exps": 16, "ffn_down_exps": 17}
ORACLE_MODEL_KINDS = {"token_embd": 0, "output_norm": 1, "output": 2}


def oracle_model(oracle, model, n_ctx):
    """The oracle's Transformer over a kestrel_b200.synth model."""
    c = model["cfg"]
    m = oracle.Model(dict(n_layer=c["n_layer"], d=c["d"], n_head=c["n_head"], n_kv=c["n_kv"],
                          head_dim=c["head_dim"], n_vocab=c["n_vocab"], n_ctx=n_ctx, rope_dim=c["rope_dim"],
                          rope_base=c["rope_base"], eps=c["eps"], arch=c["arch"], n_expert=c.get("n_expert", 0),
                          k=c.get("k", 0), norm_topk=c.get("norm_topk", True),
                          weights_scale=c.get("weights_scale", 0.0)))
    for layer, name, t, data, rows, cols in model["tensors"]:
        kind = ORACLE_MODEL_KINDS[name] if layer < 0 else ORACLE_KINDS[name]
        m.set(layer, kind, t, data, rows, cols)
    return m
