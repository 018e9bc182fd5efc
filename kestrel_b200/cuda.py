"""ctypes binding of libkestrel_cuda.so (include/kestrel_cuda.h).

The Python mirror of the calls Kestrel's engine makes on its MoE path:
`Context.moe_ffn` is Transformer::moe_ffn (crates/kestrel-engine/src/
transformer.rs:513-589), `Context.matmul` is quant::matmul (quant.rs:229-339),
`Context.upload_experts` is ExpertStore::preload_all into HBM (crates/
kestrel-memory/src/expert.rs:620-641). Failures raise `KestrelCudaError`
carrying the library's status code and message (the analogue of
EngineError, transformer.rs:15-27); there is no CPU fallback: if the CUDA
library is missing or fails to load, importing this module raises.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import ggml as G

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkestrel_cuda.so")

STATUS = {0: "OK", 1: "ERR_ARG", 2: "ERR_SHAPE", 3: "ERR_TYPE", 4: "ERR_CUDA", 5: "ERR_NCCL",
          6: "ERR_TIMEOUT", 7: "ERR_STATE", 8: "ERR_OOM"}

# Every symbol include/kestrel_cuda.h declares, with its ctypes signature.
P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
SIGNATURES = {
    "kc_init": (I, [I, ctypes.POINTER(P)]),
    "kc_free": (None, [P]),
    "kc_last_error": (ctypes.c_char_p, [P]),
    "kc_set_stream": (I, [P, P]),
    "kc_reserve": (I, [P, I]),
    "kc_sync": (I, [P]),
    "kc_device_bytes": (I64, [P]),
    "kc_upload_experts": (I, [P, I, I, I, I, I, P, I, P, I, P, I]),
    "kc_upload_experts_range": (I, [P, I, I, I, I, I, I, I, P, I, P, I, P, I]),
    "kc_upload_router": (I, [P, I, P, I, I, I, I, F, I]),
    "kc_upload_dense": (I, [P, I, I, P, I64, I64, I]),
    "kc_moe_ffn": (I, [P, I, P, I, P, I, I, I, F, P, P, P]),
    "kc_moe_ffn_dev": (I, [P, I, P, I, P, P, P]),
    "kc_matmul": (I, [P, I, P, I, P]),
    "kc_matmul_dev": (I, [P, I, P, I, P]),
    "kc_q8k_quantize_dev": (I, [P, P, I64, I64, P, P, P]),
    "kc_q8_quantize_dev": (I, [P, P, I64, I64, P, P, P]),
    "kc_route_dev": (I, [P, P, I, I, I, I, F, P, P]),
    "kc_router_logits_dev": (I, [P, P, I, I, P, I, P]),
    "kc_block_sums_dev": (I, [P, I, P, I64, I64, P, P, I, P]),
    "kc_quantize_dev": (I, [P, I, P, I64, I64, P]),
    "kc_profile_enable": (I, [P, I]),
    "kc_profile_read": (I, [P, P, P, I]),
    "kc_kernel_launches": (I64, []),
    "kc_route_noalloc": (I, [P, I, I, P, I, I, I, F, P, P, P]),
    "kc_upload_shared_expert": (I, [P, I, I, I, I, P, I, P, I, P, P, I]),
    "kc_ep_unique_id": (I, [ctypes.c_char_p]),
    "kc_ep_init": (I, [P, I, I, ctypes.c_char_p]),
    "kc_ep_reserve": (I, [P, I]),
    "kc_set_option": (I, [P, I, I]),
    "kc_model_init": (I, [P, I, I, I, I, I, I, I, I, F, F, I]),
    "kc_model_tensor": (I, [P, I, I, I, P, I64, I64, I]),
    "kc_model_forward": (I, [P, P, I, P, P]),
    "kc_model_generate": (I, [P, P, I, I, P]),
    "kc_model_generate_batch": (I, [P, I, P, P, I, P]),
    "kc_model_set_sequences": (I, [P, I]),
    "kc_model_prefill_seq": (I, [P, I, P, I, P]),
    "kc_model_decode_seqs": (I, [P, I, I, P]),
    "kc_model_truncate": (I, [P, I]),
    "kc_model_cached": (I, [P]),
    "kc_load_gguf": (I, [P, ctypes.c_char_p, I, ctypes.c_char_p, I64]),
    "kc_gguf_inspect": (I, [ctypes.c_char_p, ctypes.c_char_p, I64]),
    "kc_upload_experts_streamed": (I, [P, I, I, I, I, I, P, I, P, I, P, I]),
    "kc_expert_cache_reserve": (I, [P, I, I, I, I]),
    "kc_expert_prefetch": (I, [P, I, P, I]),
    "kc_expert_cache_stats": (I, [P, P, I]),
    "kc_expert_cache_decay": (I, [P]),
}

# Options (kc_set_option) and whole-model tensor kinds (kc_model_tensor).
OPT_F32_PREFILL = 1
OPT_LOOKAHEAD = 2
# Expert-cache policies (kc_expert_cache_reserve) and counters (kc_expert_cache_stats).
EXPERT_POLICY_LFRU, EXPERT_POLICY_LRU = 0, 1
XS_COUNTERS = ["capacity", "cached", "requests", "hits", "late", "misses", "scratch_loads", "bytes_read",
               "prefetch_issued", "prefetch_used", "prefetch_wasted", "evictions", "lookahead_predicted",
               "lookahead_correct", "reads", "forced", "scratch", "spec", "spec_pauses"]
ARCH_LLAMA, ARCH_QWEN2, ARCH_QWEN3 = 0, 1, 2
(T_ATTN_NORM, T_ATTN_Q, T_ATTN_K, T_ATTN_V, T_ATTN_OUT, T_ATTN_Q_BIAS, T_ATTN_K_BIAS, T_ATTN_V_BIAS,
 T_ATTN_Q_NORM, T_ATTN_K_NORM, T_FFN_NORM, T_FFN_GATE, T_FFN_UP, T_FFN_DOWN) = range(14)
T_TOKEN_EMBD, T_OUTPUT_NORM, T_OUTPUT = 0, 1, 2


class KestrelCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


def load_library(path: str = LIB_PATH) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m kestrel_b200.build` "
                          "(there is no CPU fallback for the CUDA path)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        _lib = load_library()
    return _lib


def _ptr(a):
    """Address of a numpy array or a torch tensor (host or device). For a
    writable numpy array the address comes through the buffer protocol
    (several times cheaper than ndarray.ctypes, which builds a helper object
    per call: it matters on the per-call path); read-only, empty or
    non-contiguous arrays take ndarray.ctypes."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        try:
            return ctypes.addressof(ctypes.c_char.from_buffer(a))
        except (TypeError, ValueError, BufferError):
            return a.ctypes.data
    return a.data_ptr()


def _is_dev(a) -> bool:
    return not isinstance(a, np.ndarray) and getattr(a, "is_cuda", False)


def _host_u8(a):
    return np.ascontiguousarray(a, dtype=np.uint8).reshape(-1) if isinstance(a, np.ndarray) else a


class Context:
    """One GPU's backend context (kc_ctx)."""

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        rc = lib().kc_init(device, ctypes.byref(h))
        if rc != 0:
            raise KestrelCudaError(rc, lib().kc_last_error(None).decode())
        self.h = h
        self.device = device
        self._k = {}           # layer -> top-k of its uploaded router
        self._dense_rows = {}  # tensor id -> rows

    def close(self):
        if getattr(self, "h", None):
            lib().kc_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int):
        if rc != 0:
            raise KestrelCudaError(rc, lib().kc_last_error(self.h).decode())

    # ---- set-up --------------------------------------------------------
    def reserve(self, max_tokens: int):
        self._check(lib().kc_reserve(self.h, max_tokens))

    def set_stream(self, stream_ptr: int | None):
        self._check(lib().kc_set_stream(self.h, stream_ptr))

    def sync(self):
        self._check(lib().kc_sync(self.h))

    def device_bytes(self) -> int:
        return int(lib().kc_device_bytes(self.h))

    def upload_experts(self, layer: int, n_expert: int, d: int, ff: int, t_gate: int, gate, t_up: int, up,
                       t_down: int, down, first_expert: int = 0, n_local: int | None = None):
        """Stacked GGUF expert tensors (numpy host bytes or torch CUDA uint8)."""
        n_local = n_expert if n_local is None else n_local
        gate, up, down = _host_u8(gate), _host_u8(up), _host_u8(down)
        dev = _is_dev(gate)
        for t, a, rows, cols in ((t_gate, gate, ff, d), (t_up, up, ff, d), (t_down, down, d, ff)):
            want = n_local * rows * G.bytes_for(t, cols)
            n = a.size if isinstance(a, np.ndarray) else a.numel() * a.element_size()
            if n < want:
                raise ValueError(f"expert tensor holds {n} bytes, {want} needed")
        self._check(lib().kc_upload_experts_range(self.h, layer, n_expert, first_expert, n_local, d, ff, t_gate,
                                                  _ptr(gate), t_up, _ptr(up), t_down, _ptr(down), int(dev)))

    def upload_experts_streamed(self, layer: int, n_expert: int, d: int, ff: int, t_gate: int, gate, t_up: int,
                                up, t_down: int, down):
        """Like upload_experts, but the experts stay in pinned host memory and
        each call copies the ones it routes to into HBM slots."""
        gate, up, down = _host_u8(gate), _host_u8(up), _host_u8(down)
        dev = _is_dev(gate)
        for t, a, rows, cols in ((t_gate, gate, ff, d), (t_up, up, ff, d), (t_down, down, d, ff)):
            want = n_expert * rows * G.bytes_for(t, cols)
            n = a.size if isinstance(a, np.ndarray) else a.numel() * a.element_size()
            if n < want:
                raise ValueError(f"expert tensor holds {n} bytes, {want} needed")
        self._check(lib().kc_upload_experts_streamed(self.h, layer, n_expert, d, ff, t_gate, _ptr(gate), t_up,
                                                     _ptr(up), t_down, _ptr(down), int(dev)))

    def expert_cache_reserve(self, capacity: int, scratch: int = 0, policy: int = EXPERT_POLICY_LFRU,
                             spec: int | None = None):
        """spec: speculative slots (default max(1, scratch), as ExpertStore::new sets)."""
        spec = max(1, scratch) if spec is None else spec
        self._check(lib().kc_expert_cache_reserve(self.h, capacity, scratch, spec, policy))

    def expert_prefetch(self, layer: int, experts):
        ids = np.ascontiguousarray(np.asarray(experts, dtype=np.int32))
        self._check(lib().kc_expert_prefetch(self.h, layer, ids.ctypes.data, ids.size))

    def expert_cache_stats(self) -> dict:
        out = np.zeros(len(XS_COUNTERS), np.uint64)
        self._check(lib().kc_expert_cache_stats(self.h, out.ctypes.data, out.size))
        return {k: int(v) for k, v in zip(XS_COUNTERS, out)}

    def expert_cache_decay(self):
        self._check(lib().kc_expert_cache_decay(self.h))

    def upload_router(self, layer: int, router_w, k: int, norm_topk: bool = True, weights_scale: float = 0.0):
        rw = router_w if _is_dev(router_w) else np.ascontiguousarray(router_w, dtype=np.float32)
        E, d = rw.shape
        self._check(lib().kc_upload_router(self.h, layer, _ptr(rw), E, d, k, int(norm_topk), weights_scale,
                                           int(_is_dev(rw))))
        self._k[layer] = k

    def upload_shared_expert(self, layer: int, ff: int, d: int, t_gate: int, gate, t_up: int, up, t_down: int,
                             down, gate_inp=None):
        """qwen2moe shared expert of `layer` (host numpy GGUF bytes or torch CUDA
        uint8); gate_inp: optional F32 [d] gate vector."""
        gate, up, down = _host_u8(gate), _host_u8(up), _host_u8(down)
        dev = _is_dev(gate)
        gi = None if gate_inp is None else (gate_inp if _is_dev(gate_inp) else
                                            np.ascontiguousarray(gate_inp, dtype=np.float32))
        self._check(lib().kc_upload_shared_expert(self.h, layer, ff, d, t_gate, _ptr(gate), t_up, _ptr(up), t_down,
                                                  _ptr(down), _ptr(gi), int(dev)))

    def upload_dense(self, tensor_id: int, t: int, w, rows: int, cols: int):
        w = _host_u8(w) if t != G.F32 or not isinstance(w, np.ndarray) else \
            np.ascontiguousarray(w, dtype=np.float32)
        self._check(lib().kc_upload_dense(self.h, tensor_id, t, _ptr(w), rows, cols, int(_is_dev(w))))
        self._dense_rows[tensor_id] = rows

    # ---- hot path (host buffers) -------------------------------------------
    def moe_ffn(self, layer: int, h, router_w=None, k: int = 0, norm_topk: bool = True,
                weights_scale: float = 0.0, out=None, topk: bool = True):
        """Transformer::moe_ffn on host f32 h [n, d] -> (out, topk ids, topk w).
        `out`: optional caller buffer (e.g. pinned) for the result; with
        topk=False the ids and weights are not copied back (returned as None)."""
        h = np.ascontiguousarray(h, dtype=np.float32)
        n, d = h.shape
        rw = None if router_w is None else np.ascontiguousarray(router_w, dtype=np.float32)
        E = 0 if rw is None else rw.shape[0]
        kk = k if rw is not None else self._layer_k(layer)
        if out is None:
            out = np.empty((n, d), np.float32)
        elif out.dtype != np.float32 or out.shape != (n, d) or not out.flags.c_contiguous:
            raise ValueError("out must be a C-contiguous float32 [n, d] array")
        ids = np.empty((n, kk), np.int32) if topk else None
        w = np.empty((n, kk), np.float32) if topk else None
        self._check(lib().kc_moe_ffn(self.h, layer, _ptr(h), n, _ptr(rw), E, k, int(norm_topk), weights_scale,
                                     _ptr(out), _ptr(ids), _ptr(w)))
        return out, ids, w

    def _layer_k(self, layer):
        if layer not in self._k:
            raise ValueError("router not uploaded through this Context; pass router_w and k")
        return self._k[layer]

    def matmul(self, tensor_id: int, x) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows = self._dense_rows[tensor_id]
        out = np.empty((x.shape[0], rows), np.float32)
        self._check(lib().kc_matmul(self.h, tensor_id, _ptr(x), x.shape[0], _ptr(out)))
        return out

    # ---- device buffers (torch CUDA tensors) ---------------------------------
    def moe_ffn_dev(self, layer: int, h, out, ids=None, w=None, n_tok: int | None = None):
        n = h.shape[0] if n_tok is None else n_tok
        self._check(lib().kc_moe_ffn_dev(self.h, layer, _ptr(h), n, _ptr(out), _ptr(ids), _ptr(w)))

    def matmul_dev(self, tensor_id: int, x, out, n: int | None = None):
        self._check(lib().kc_matmul_dev(self.h, tensor_id, _ptr(x), x.shape[0] if n is None else n, _ptr(out)))

    def q8k_quantize_dev(self, x, q, d, bsums):
        self._check(lib().kc_q8k_quantize_dev(self.h, _ptr(x), x.shape[0], x.shape[1], _ptr(q), _ptr(d),
                                              _ptr(bsums)))

    def q8_quantize_dev(self, x, q, d, s16):
        self._check(lib().kc_q8_quantize_dev(self.h, _ptr(x), x.shape[0], x.shape[1], _ptr(q), _ptr(d),
                                             _ptr(s16)))

    def route_dev(self, logits, k: int, ids, w, norm_topk: bool = True, weights_scale: float = 0.0):
        n, E = logits.shape
        self._check(lib().kc_route_dev(self.h, _ptr(logits), n, E, k, int(norm_topk), weights_scale, _ptr(ids),
                                       _ptr(w)))

    def router_logits_dev(self, router_w, h, logits):
        E, d = router_w.shape
        self._check(lib().kc_router_logits_dev(self.h, _ptr(router_w), E, d, _ptr(h), h.shape[0], _ptr(logits)))

    def block_sums_dev(self, t: int, w, rows: int, cols: int, q, bsums, n_act: int, out):
        self._check(lib().kc_block_sums_dev(self.h, t, _ptr(w), rows, cols, _ptr(q), _ptr(bsums), n_act,
                                            _ptr(out)))

    def quantize_dev(self, t: int, x, out):
        rows, cols = x.shape
        self._check(lib().kc_quantize_dev(self.h, t, _ptr(x), rows, cols, _ptr(out)))

    STAGES = ["router_logits", "route", "dispatch", "quant_x", "gate_up_int8", "gate_up_f32", "quant_act",
              "down_int8", "down_f32", "combine", "expert_load"]

    def profile_enable(self, on: bool = True):
        self._check(lib().kc_profile_enable(self.h, int(on)))

    def profile_read(self) -> dict:
        """{stage: (total ms, calls)} accumulated since the previous read."""
        n = len(self.STAGES)
        ms = np.zeros(n, np.float64)
        calls = np.zeros(n, np.int64)
        self._check(lib().kc_profile_read(self.h, ms.ctypes.data, calls.ctypes.data, n))
        return {s: (float(ms[i]), int(calls[i])) for i, s in enumerate(self.STAGES)}

    def ep_init(self, rank: int, world: int, uid: bytes):
        self._check(lib().kc_ep_init(self.h, rank, world, uid))

    # ---- whole model (dense decode path) ---------------------------------------
    def set_option(self, option: int, value: int):
        self._check(lib().kc_set_option(self.h, option, int(value)))

    def model_init(self, n_layer: int, d: int, n_head: int, n_head_kv: int, head_dim: int, n_vocab: int,
                   n_ctx: int, rope_dim: int, rope_base: float, rms_eps: float, arch: int):
        self._n_vocab = n_vocab
        self._check(lib().kc_model_init(self.h, n_layer, d, n_head, n_head_kv, head_dim, n_vocab, n_ctx, rope_dim,
                                        rope_base, rms_eps, arch))

    def model_tensor(self, layer: int, kind: int, t: int, w, rows: int, cols: int):
        """A model tensor (layer -1) or a layer tensor; host numpy bytes / f32
        or a torch CUDA tensor."""
        if _is_dev(w):
            self._check(lib().kc_model_tensor(self.h, layer, kind, t, _ptr(w), rows, cols, 1))
            return
        a = np.ascontiguousarray(w, dtype=np.float32) if t == G.F32 else _host_u8(w)
        self._check(lib().kc_model_tensor(self.h, layer, kind, t, _ptr(a), rows, cols, 0))

    def model_forward(self, tokens):
        """Transformer::forward: logits of the last token (and its argmax)."""
        tk = np.ascontiguousarray(tokens, dtype=np.uint32)
        logits = np.empty(self._n_vocab, np.float32)
        nxt = np.zeros(1, np.uint32)
        self._check(lib().kc_model_forward(self.h, _ptr(tk), tk.size, _ptr(logits), _ptr(nxt)))
        return logits, int(nxt[0])

    def model_generate(self, prompt, n_gen: int):
        tk = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.zeros(max(1, n_gen), np.uint32)
        self._check(lib().kc_model_generate(self.h, _ptr(tk), tk.size, n_gen, _ptr(out)))
        return [int(t) for t in out[:n_gen]]

    def model_generate_batch(self, prompts, n_gen: int):
        """kc_model_generate_batch: greedy decode of len(prompts) independent
        sequences in lockstep; returns one token list per sequence."""
        lens = np.array([len(p) for p in prompts], dtype=np.int32)
        flat = np.ascontiguousarray(np.concatenate([np.asarray(p, dtype=np.uint32) for p in prompts]))
        out = np.zeros((len(prompts), max(1, n_gen)), np.uint32)
        self._check(lib().kc_model_generate_batch(self.h, len(prompts), _ptr(flat), _ptr(lens), n_gen, _ptr(out)))
        return [[int(t) for t in row[:n_gen]] for row in out]

    def model_set_sequences(self, n_seq: int):
        self._check(lib().kc_model_set_sequences(self.h, n_seq))

    def model_prefill_seq(self, seq: int, prompt) -> int:
        """kc_model_prefill_seq: the prompt alone in sequence `seq`'s cache;
        returns its greedy next token (the sequence's pending token)."""
        tk = np.ascontiguousarray(prompt, dtype=np.uint32)
        nxt = np.zeros(1, np.uint32)
        self._check(lib().kc_model_prefill_seq(self.h, seq, _ptr(tk), tk.size, _ptr(nxt)))
        return int(nxt[0])

    def model_decode_seqs(self, n_seq: int, n_gen: int):
        out = np.zeros((n_seq, max(1, n_gen)), np.uint32)
        self._check(lib().kc_model_decode_seqs(self.h, n_seq, n_gen, _ptr(out)))
        return [[int(t) for t in row[:n_gen]] for row in out]

    def model_truncate(self, keep: int):
        self._check(lib().kc_model_truncate(self.h, keep))

    def model_cached(self) -> int:
        return int(lib().kc_model_cached(self.h))

    def load_gguf(self, path: str, n_ctx: int) -> dict:
        """kc_load_gguf: declare and upload a GGUF / KGUF model; returns the
        loader's summary (weight, KV-cache and free bytes)."""
        import json
        buf = ctypes.create_string_buffer(4096)
        rc = lib().kc_load_gguf(self.h, os.fsencode(path), n_ctx, buf, len(buf))
        info = json.loads(buf.value.decode()) if buf.value else {}
        self._check(rc)
        self._n_vocab = int(info.get("n_vocab", getattr(self, "_n_vocab", 0)))
        return info

    def ep_reserve(self, max_tokens: int):
        """Collective: map the peer exchange arenas for up to max_tokens tokens
        per rank and call (after uploading the layers)."""
        self._check(lib().kc_ep_reserve(self.h, max_tokens))


def gguf_inspect(path: str) -> dict:
    """kc_gguf_inspect: parse a GGUF / KGUF file (no GPU needed)."""
    import json
    cap = 1 << 22
    buf = ctypes.create_string_buffer(cap)
    rc = lib().kc_gguf_inspect(os.fsencode(path), buf, cap)
    if rc != 0:
        raise KestrelCudaError(rc, (lib().kc_last_error(None) or b"").decode())
    return json.loads(buf.value.decode())


def ep_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    rc = lib().kc_ep_unique_id(buf)
    if rc != 0:
        raise KestrelCudaError(rc, "ncclGetUniqueId failed")
    return buf.raw


def kernel_launches() -> int:
    """CUDA kernels this library has launched in the process so far
    (kc_kernel_launches)."""
    return int(lib().kc_kernel_launches())
