"""TEST INFRASTRUCTURE ONLY -- the parity checker, never the product.

ctypes bindings for `libkestrel_oracle.so`, the C++ restatement of Kestrel's
CPU arithmetic on the MoE FFN path (kestrel_oracle.cpp cites the reference
lines each function follows). Only tests/, `__graft_entry__.smoke()` and the
CPU legs of bench.py may import this package.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkestrel_oracle.so")

_lib = None


def build() -> str:
    """Compile the oracle library (make; seconds)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "kestrel_oracle.cpp")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, I, F = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        sig = {
            "ko_set_threads": (None, [I]), "ko_get_threads": (I, []),
            "ko_block_elems": (I, [I]), "ko_block_bytes": (I, [I]), "ko_bytes_for": (I64, [I, I64]),
            "ko_f16_to_f32": (F, [ctypes.c_uint16]),
            "ko_dequant_row": (None, [I, P, I64, P]),
            "ko_dot": (F, [P, P, I64]), "ko_dot_f32": (F, [P, P, I64]), "ko_lane_chain_f32": (F, [P, P, I64]),
            "ko_gemm_f32": (None, [P, I64, P, I64, I64, P]),
            "ko_q8_quantize": (None, [P, I64, P, P, P]), "ko_q8k_quantize": (None, [P, I64, P, P, P]),
            "ko_unpack": (None, [I, P, I64, P, P, P]),
            "ko_dot_unpacked": (F, [P, P, P, I64, P, P, P]),
            "ko_dot_unpacked_scalar": (F, [P, P, P, I64, P, P, P]),
            "ko_dot_fused": (F, [I, P, I64, P, P, P]), "ko_dot_q8_0_lanes": (F, [P, I64, P, P]),
            "ko_dot_fused_k": (F, [I, P, I64, P, P, P, I]),
            "ko_block_sums_k": (None, [I, P, I64, P, P, P]),
            "ko_set_exact": (None, [I]),
            "ko_matmul": (I, [I, P, I64, I64, P, I64, P]),
            "ko_route": (None, [P, I64, I, I, I, F, P, P]),
            "ko_moe_ffn": (I, [P, I64, I64, P, I, I, I, F, I, P, I, P, I, P, I64, P, P, P,
                               I, P, I, P, I, P, I64, P]),
            "ko_argmax": (I, [P, I64]),
            "ko_expert_ffn": (I, [I, P, I, P, I, P, I64, I64, P, I64, P]),
            "ko_model_new": (P, [I, I, I, I, I, I, I, I, F, F, I, I, I, I, F]),
            "ko_model_free": (None, [P]),
            "ko_model_set": (I, [P, I, I, I, P, I64, I64]),
            "ko_model_forward": (I, [P, P, I, P]),
            "ko_model_truncate": (None, [P, I]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8).reshape(-1)


def set_threads(n: int) -> None:
    lib().ko_set_threads(int(n))


def set_exact(on: bool) -> None:
    lib().ko_set_exact(1 if on else 0)


def dequant_row(t: int, src, n: int) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    s = _u8(src)
    lib().ko_dequant_row(t, _p(s), n, _p(out))
    return out


def dequant(t: int, w, rows: int, cols: int) -> np.ndarray:
    """Dequantize a `[rows, cols]` matrix (row by row, dequant_row)."""
    wb = _u8(w).reshape(rows, -1)
    return np.stack([dequant_row(t, wb[r], cols) for r in range(rows)]) if rows else np.zeros((0, cols), np.float32)


def q8k_quantize(x):
    x = _f32(x).reshape(-1)
    n = x.size
    q = np.empty(n, np.int8)
    d = np.empty(n // 256, np.float32)
    bs = np.empty(n // 16, np.int32)
    lib().ko_q8k_quantize(_p(x), n, _p(q), _p(d), _p(bs))
    return q, d, bs


def q8_quantize(x):
    x = _f32(x).reshape(-1)
    n = x.size
    q = np.empty(n, np.int8)
    d = np.empty(n // 32, np.float32)
    s16 = np.empty(n // 16, np.int32)
    lib().ko_q8_quantize(_p(x), n, _p(q), _p(d), _p(s16))
    return q, d, s16


def unpack(t: int, w, n: int):
    q = np.empty(n, np.int8)
    sc = np.empty(n // 16, np.float32)
    mn = np.empty(n // 16, np.float32)
    wb = _u8(w)
    lib().ko_unpack(t, _p(wb), n, _p(q), _p(sc), _p(mn))
    return q, sc, mn


def dot(a, b) -> float:
    a, b = _f32(a), _f32(b)
    return float(lib().ko_dot(_p(a), _p(b), a.size))


def dot_f32(a, b) -> float:
    a, b = _f32(a), _f32(b)
    return float(lib().ko_dot_f32(_p(a), _p(b), a.size))


def lane_chain_f32(a, b) -> float:
    a, b = _f32(a), _f32(b)
    return float(lib().ko_lane_chain_f32(_p(a), _p(b), a.size))


def gemm_f32(w, rows: int, x, s_rows: int, cols: int) -> np.ndarray:
    w, x = _f32(w), _f32(x)
    res = np.empty(rows * s_rows, np.float32)
    lib().ko_gemm_f32(_p(w), rows, _p(x), s_rows, cols, _p(res))
    return res.reshape(rows, s_rows)


def dot_unpacked(uq, usc, umn, q, d, s16, scalar: bool = False) -> float:
    f = lib().ko_dot_unpacked_scalar if scalar else lib().ko_dot_unpacked
    return float(f(_p(uq), _p(usc), _p(umn), uq.size, _p(q), _p(d), _p(s16)))


def dot_fused(t: int, w, q, d, s16) -> float:
    wb = _u8(w)
    return float(lib().ko_dot_fused(t, _p(wb), q.size, _p(q), _p(d), _p(s16)))


def dot_q8_0_lanes(w, q, d) -> float:
    wb = _u8(w)
    return float(lib().ko_dot_q8_0_lanes(_p(wb), q.size, _p(q), _p(d)))


def dot_fused_k(t: int, w, q, d, bsums, lanes: bool = False) -> float:
    wb = _u8(w)
    return float(lib().ko_dot_fused_k(t, _p(wb), q.size, _p(q), _p(d), _p(bsums), 1 if lanes else 0))


def block_sums_k(t: int, w, q, bsums) -> np.ndarray:
    """[n/256, 9] int32: the eight lanes of sumi and the min/offset term."""
    wb = _u8(w)
    out = np.empty((q.size // 256, 9), np.int32)
    lib().ko_block_sums_k(t, _p(wb), q.size, _p(q), _p(bsums), _p(out))
    return out


def matmul(t: int, w, rows: int, cols: int, x) -> np.ndarray:
    """quant::matmul: x [S, cols] f32 -> out [S, rows] f32."""
    wb = _u8(w)
    x = _f32(x).reshape(-1, cols)
    out = np.empty((x.shape[0], rows), np.float32)
    rc = lib().ko_matmul(t, _p(wb), rows, cols, _p(x), x.shape[0], _p(out))
    if rc:
        raise ValueError(f"oracle matmul rejected type {t} cols {cols}")
    return out


def route(logits, k: int, norm_topk: bool = True, weights_scale: float = 0.0):
    lg = _f32(logits)
    n, E = lg.shape
    ids = np.empty((n, k), np.int32)
    w = np.empty((n, k), np.float32)
    lib().ko_route(_p(lg), n, E, k, 1 if norm_topk else 0, weights_scale, _p(ids), _p(w))
    return ids, w


def moe_ffn(h, router_w, k: int, t_gate: int, gate, t_up: int, up, t_down: int, down, ff: int,
            norm_topk: bool = True, weights_scale: float = 0.0, shared=None):
    """Transformer::moe_ffn for one layer. h [S, d] f32; router_w [E, d] f32;
    gate/up/down: stacked GGUF bytes of all experts. `shared` is an optional
    dict(t_gate, gate, t_up, up, t_down, down, ff, inp) for the qwen2moe shared
    expert. Returns (out [S, d], topk ids [S, k], topk weights [S, k])."""
    h = _f32(h)
    n, d = h.shape
    rw = _f32(router_w)
    E = rw.shape[0]
    out = np.empty((n, d), np.float32)
    ids = np.empty((n, k), np.int32)
    w = np.empty((n, k), np.float32)
    g, u, dn = _u8(gate), _u8(up), _u8(down)
    sh = shared or {}
    shg = _u8(sh["gate"]) if sh else None
    shu = _u8(sh["up"]) if sh else None
    shd = _u8(sh["down"]) if sh else None
    shi = _f32(sh["inp"]) if sh.get("inp") is not None else None
    rc = lib().ko_moe_ffn(
        _p(h), n, d, _p(rw), E, k, 1 if norm_topk else 0, weights_scale,
        t_gate, _p(g), t_up, _p(u), t_down, _p(dn), ff, _p(out), _p(ids), _p(w),
        sh.get("t_gate", 0), _p(shg), sh.get("t_up", 0), _p(shu), sh.get("t_down", 0), _p(shd),
        sh.get("ff", 0), _p(shi))
    if rc:
        raise ValueError("oracle moe_ffn rejected its arguments")
    return out, ids, w


def expert_ffn(t_gate: int, gate_e, t_up: int, up_e, t_down: int, down_e, d: int, ff: int, xs) -> np.ndarray:
    """One expert of moe_ffn on its rows xs [n, d] (transformer.rs:551-563):
    gate/up products, SwiGLU, down product -> [n, d]. gate_e / up_e / down_e
    are that expert's GGUF bytes ([ff] rows of d, [d] rows of ff)."""
    xs = _f32(xs).reshape(-1, d)
    y = np.empty((xs.shape[0], d), np.float32)
    g, u, dn = _u8(gate_e), _u8(up_e), _u8(down_e)
    rc = lib().ko_expert_ffn(t_gate, _p(g), t_up, _p(u), t_down, _p(dn), d, ff, _p(xs), xs.shape[0], _p(y))
    if rc:
        raise ValueError("oracle expert_ffn rejected the shapes")
    return y


def argmax(logits) -> int:
    lg = _f32(logits)
    return int(lib().ko_argmax(_p(lg), lg.size))


class Model:
    """Transformer::forward (transformer.rs:287-467) over host weights.

    hp: n_layer, d, n_head, n_kv, head_dim, n_vocab, n_ctx, rope_dim,
    rope_base, eps, arch (0 llama, 1 qwen2, 2 qwen3), n_expert, k, norm_topk,
    weights_scale. Tensors are (layer, kind, ggml type, bytes or f32 array,
    rows, cols); layer -1 for the model tensors (embedding, output norm,
    output)."""

    def __init__(self, hp: dict):
        self.hp = dict(hp)
        L = lib()
        self._h = L.ko_model_new(hp["n_layer"], hp["d"], hp["n_head"], hp["n_kv"], hp["head_dim"], hp["n_vocab"],
                                 hp["n_ctx"], hp["rope_dim"], hp["rope_base"], hp["eps"], hp["arch"],
                                 hp.get("n_expert", 0), hp.get("k", 0), 1 if hp.get("norm_topk", True) else 0,
                                 hp.get("weights_scale", 0.0))
        self._keep = []

    def set(self, layer: int, kind: int, t: int, w, rows: int, cols: int) -> None:
        a = np.ascontiguousarray(w)
        self._keep.append(a)
        if lib().ko_model_set(self._h, layer, kind, t, a.ctypes.data, rows, cols):
            raise ValueError(f"oracle model rejected tensor kind {kind} of layer {layer}")

    def forward(self, tokens) -> np.ndarray:
        tk = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.hp["n_vocab"], np.float32)
        rc = lib().ko_model_forward(self._h, tk.ctypes.data, tk.size, out.ctypes.data)
        if rc:
            raise ValueError(f"oracle forward failed ({rc})")
        return out

    def truncate(self, keep: int) -> None:
        lib().ko_model_truncate(self._h, keep)

    def generate(self, prompt, n_gen: int):
        """Greedy decode (crates/kestrel-engine/src/lib.rs:116-145 with
        SamplerConfig::greedy): returns n_gen tokens and the logits each was
        taken from."""
        logits = self.forward(prompt)
        toks, all_logits = [], []
        for i in range(n_gen):
            t = int(lib().ko_argmax(logits.ctypes.data, logits.size))
            toks.append(t)
            all_logits.append(logits)
            if i + 1 == n_gen:
                break
            logits = self.forward([t])
        return toks, all_logits

    def __del__(self):
        try:
            lib().ko_model_free(self._h)
        except Exception:
            pass
