"""The oracle's Transformer::forward restatement against an independent
float64 numpy forward of the same model (structure: head layout, GQA
grouping, RoPE pairing, q/k norms, biases, residuals, routed and dense FFN,
KV cache across calls). The numpy forward rounds nothing, so agreement is to
within float32 rounding, not bit for bit; the oracle's arithmetic itself is
pinned by the kernel-level tests and golden vectors."""
import numpy as np
import pytest

import oracle
from kestrel_b200 import ggml as G
from kestrel_b200 import synth
from gpu_util import oracle_model


def np_forward(model, tokens_list):
    """Float64 forward over the dequantised weights; returns the last-token
    logits after each call in tokens_list (the KV cache carries over)."""
    c = model["cfg"]
    T = {}
    for layer, name, t, data, rows, cols in model["tensors"]:
        T[(layer, name)] = (oracle.dequant(t, data, rows, cols) if t != G.F32 else
                            np.asarray(data, np.float32).reshape(rows, cols)).astype(np.float64)
    d, nh, nkv, hd, rd = c["d"], c["n_head"], c["n_kv"], c["head_dim"], c["rope_dim"]
    inv = np.array([np.float32(c["rope_base"]) ** (-(2.0 * i) / rd) for i in range(rd // 2)])
    neox = c["arch"] != synth.ARCH_LLAMA

    def norm(x, w, eps=c["eps"]):
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w.reshape(-1)

    def rope(v, pos):
        out = v.copy()
        for i in range(rd // 2):
            a, b = (i, i + rd // 2) if neox else (2 * i, 2 * i + 1)
            s, co = np.sin(pos * inv[i]), np.cos(pos * inv[i])
            out[..., a] = v[..., a] * co - v[..., b] * s
            out[..., b] = v[..., a] * s + v[..., b] * co
        return out

    K = [np.zeros((0, nkv, hd)) for _ in range(c["n_layer"])]
    V = [np.zeros((0, nkv, hd)) for _ in range(c["n_layer"])]
    pos0, results = 0, []
    for toks in tokens_list:
        n = len(toks)
        x = T[(-1, "token_embd")][toks]
        for l in range(c["n_layer"]):
            h = norm(x, T[(l, "attn_norm")])
            q = (h @ T[(l, "attn_q")].T).reshape(n, nh, hd)
            k = (h @ T[(l, "attn_k")].T).reshape(n, nkv, hd)
            v = (h @ T[(l, "attn_v")].T).reshape(n, nkv, hd)
            if (l, "attn_q_bias") in T:
                q += T[(l, "attn_q_bias")].reshape(nh, hd)
                k += T[(l, "attn_k_bias")].reshape(nkv, hd)
                v += T[(l, "attn_v_bias")].reshape(nkv, hd)
            if (l, "attn_q_norm") in T:
                q, k = norm(q, T[(l, "attn_q_norm")]), norm(k, T[(l, "attn_k_norm")])
            pos = np.arange(pos0, pos0 + n, dtype=np.float64)[:, None]
            q, k = rope(q, pos), rope(k, pos)
            K[l] = np.concatenate([K[l], k.astype(np.float16).astype(np.float64)])
            V[l] = np.concatenate([V[l], v.astype(np.float16).astype(np.float64)])
            att = np.zeros((n, nh, hd))
            for s in range(n):
                for hh in range(nh):
                    kv = hh // (nh // nkv)
                    sc = K[l][:pos0 + s + 1, kv] @ q[s, hh] / np.sqrt(hd)
                    p = np.exp(sc - sc.max())
                    att[s, hh] = (p / p.sum()) @ V[l][:pos0 + s + 1, kv]
            x = x + att.reshape(n, -1) @ T[(l, "attn_output")].T
            h = norm(x, T[(l, "ffn_norm")])
            if (l, "ffn_gate_inp") in T:
                E, k_, ff = c["n_expert"], c["k"], c["ff"]
                lg = h @ T[(l, "ffn_gate_inp")].T
                p = np.exp(lg - lg.max(-1, keepdims=True))
                p /= p.sum(-1, keepdims=True)
                y = np.zeros_like(x)
                for s in range(n):
                    sel = np.argsort(-p[s], kind="stable")[:k_]
                    wts = p[s, sel] / (p[s, sel].sum() if c["norm_topk"] else 1.0)
                    for e, wt in zip(sel, wts):
                        g = T[(l, "ffn_gate_exps")][e * ff:(e + 1) * ff] @ h[s]
                        u = T[(l, "ffn_up_exps")][e * ff:(e + 1) * ff] @ h[s]
                        a = g / (1 + np.exp(-g)) * u
                        y[s] += wt * (T[(l, "ffn_down_exps")][e * d:(e + 1) * d] @ a)
            else:
                g, u = h @ T[(l, "ffn_gate")].T, h @ T[(l, "ffn_up")].T
                y = (g / (1 + np.exp(-g)) * u) @ T[(l, "ffn_down")].T
            x = x + y
        pos0 += n
        results.append(norm(x[-1:], T[(-1, "output_norm")]) @ T[(-1, "output")].T)
    return [r.reshape(-1) for r in results]


SMALL = dict(synth.CONFIG0, n_layer=2, d=256, n_head=4, n_kv=2, head_dim=32, rope_dim=32, n_vocab=512, ff=256,
             t_down=G.Q8_0)


@pytest.mark.parametrize("variant", ["qwen3-moe", "llama-moe", "qwen2-dense"])
def test_oracle_forward_matches_float64(variant):
    cfg = dict(SMALL)
    if variant == "llama-moe":
        cfg["arch"] = synth.ARCH_LLAMA
    if variant == "qwen2-dense":
        cfg.update(arch=synth.ARCH_QWEN2, dense_ff=512, t_gate=G.Q4_K, t_down=G.Q6_K)
    model = synth.make_model(cfg, seed=3)
    rng = np.random.default_rng(4)
    calls = [list(rng.integers(0, cfg["n_vocab"], 7)), [5], [int(rng.integers(0, cfg["n_vocab"]))]]
    ref = np_forward(model, calls)
    # exact: every product on dequantised f32 weights (no Q8 activation
    # rounding), so only float32 rounding separates the two; otherwise the
    # reference's dispatch runs the int8 path for products with < 4 rows,
    # whose activation quantisation moves logits by ~1e-2 of their scale.
    for exact, tol in ((True, 2e-6), (False, 3e-2)):
        oracle.set_exact(exact)
        try:
            m = oracle_model(oracle, model, n_ctx=32)
            for toks, r in zip(calls, ref):
                got = m.forward(toks)
                scale = max(float(np.abs(r).max()), 1.0)
                assert np.abs(got - r).max() <= tol * scale, (variant, exact, np.abs(got - r).max(), scale)
        finally:
            oracle.set_exact(False)


def test_oracle_truncate_and_generate_deterministic():
    model = synth.make_model(SMALL, seed=5)
    m = oracle_model(oracle, model, n_ctx=64)
    prompt = list(range(1, 12))
    m.forward(prompt[:-1])
    a = m.forward(prompt[-1:])
    m.forward([3, 4])
    m.truncate(len(prompt) - 1)
    b = m.forward(prompt[-1:])
    assert np.array_equal(a, b)  # same KV prefix, same last token, same (1-row) arithmetic
    m.truncate(0)
    t1, _ = m.generate(prompt, 6)
    m.truncate(0)
    t2, _ = m.generate(prompt, 6)
    assert t1 == t2 and len(t1) == 6
