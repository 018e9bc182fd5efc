"""Write GGUF v3 (and Kestrel-prepared KGUF) model files.

The container format kestrel-gguf reads (crates/kestrel-gguf/src/lib.rs:
196-311, writer.rs): magic, version 3, tensor and key/value counts, the
metadata table, the tensor infos (name, dims with dims[0] the row length,
ggml type, offset relative to the data section), then the data section
aligned to `general.alignment` (32) with every tensor aligned. A prepared
container (`KGUF` magic) may store a stacked tensor's outermost slices
`stride` bytes apart (`kestrel.stride.<name>` metadata, TensorInfo::
slice_offset, lib.rs:183-189).

`write_model` turns a kestrel_b200.synth model into a file with the metadata
keys kestrel-model reads (crates/kestrel-model/src/lib.rs:170-215, 338-373),
so that `cuda.Context.load_gguf` (kc_load_gguf) can load it.
"""
from __future__ import annotations

import struct

import numpy as np

from . import ggml as G
from . import synth

ALIGN = 32
# GGUF value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vt: int, v) -> bytes:
    fmt = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
           I64: "<q", F64: "<d"}
    if vt == STRING:
        return _str(v)
    if vt == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    return struct.pack(fmt[vt], int(v) if vt == BOOL else v)


def write_gguf(path: str, metadata: list, tensors: list, prepared: bool = False, strides: dict | None = None):
    """metadata: [(key, value type, value)]; tensors: [(name, ggml type, dims
    (ggml order), bytes)]. strides: {name: stride} for a prepared container
    (the tensor's outermost slices stored `stride` bytes apart)."""
    strides = dict(strides or {})
    meta = list(metadata) + [(f"kestrel.stride.{n}", U64, s) for n, s in strides.items()]
    layout, off = [], 0
    for name, t, dims, data in tensors:
        data = np.ascontiguousarray(data).reshape(-1).view(np.uint8)
        if name in strides:
            n_sl = dims[-1]
            sb = data.size // n_sl
            span = (n_sl - 1) * strides[name] + sb
        else:
            span = data.size
        layout.append((name, t, dims, data, off))
        off = (off + span + ALIGN - 1) // ALIGN * ALIGN
    head = bytearray(b"KGUF" if prepared else b"GGUF")
    head += struct.pack("<IQQ", 3, len(tensors), len(meta))
    for k, vt, v in meta:
        head += _str(k) + struct.pack("<I", vt) + _value(vt, v)
    for name, t, dims, data, o in layout:
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", t, o)
    data_start = (len(head) + ALIGN - 1) // ALIGN * ALIGN
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (data_start - len(head)))
        for name, t, dims, data, o in layout:
            f.seek(data_start + o)
            if name in strides:
                n_sl = dims[-1]
                sb = data.size // n_sl
                for s in range(n_sl):
                    f.seek(data_start + o + s * strides[name])
                    f.write(data[s * sb:(s + 1) * sb].tobytes())
            else:
                f.write(data.tobytes())
        end = data_start + off
        f.seek(0, 2)
        if f.tell() < end:
            f.write(b"\0" * (end - f.tell()))


ARCH_NAMES = {(synth.ARCH_LLAMA, True): "llama", (synth.ARCH_LLAMA, False): "llama",
              (synth.ARCH_QWEN2, True): "qwen2moe", (synth.ARCH_QWEN2, False): "qwen2",
              (synth.ARCH_QWEN3, True): "qwen3moe", (synth.ARCH_QWEN3, False): "qwen3"}


def write_model(path: str, model: dict, prepared: bool = False, n_ctx_train: int = 4096):
    """A kestrel_b200.synth model as a GGUF (or, prepared=True, a KGUF whose
    stacked expert tensors are strided with one alignment unit of padding
    between slices)."""
    c = model["cfg"]
    moe = not c.get("dense_ff", 0)
    arch = ARCH_NAMES[(c["arch"], moe)]
    meta = [("general.architecture", STRING, arch), ("general.alignment", U32, ALIGN),
            (f"{arch}.block_count", U32, c["n_layer"]), (f"{arch}.embedding_length", U32, c["d"]),
            (f"{arch}.attention.head_count", U32, c["n_head"]),
            (f"{arch}.attention.head_count_kv", U32, c["n_kv"]),
            (f"{arch}.attention.key_length", U32, c["head_dim"]),
            (f"{arch}.attention.value_length", U32, c["head_dim"]),
            (f"{arch}.rope.dimension_count", U32, c["rope_dim"]),
            (f"{arch}.rope.freq_base", F32, c["rope_base"]),
            (f"{arch}.attention.layer_norm_rms_epsilon", F32, c["eps"]),
            (f"{arch}.context_length", U32, n_ctx_train),
            (f"{arch}.feed_forward_length", U32, c.get("dense_ff") or c["ff"])]
    if moe:
        meta += [(f"{arch}.expert_count", U32, c["n_expert"]), (f"{arch}.expert_used_count", U32, c["k"]),
                 (f"{arch}.expert_feed_forward_length", U32, c["ff"]),
                 (f"{arch}.expert_weights_norm", BOOL, bool(c["norm_topk"]))]
        if c.get("weights_scale", 0.0):
            meta.append((f"{arch}.expert_weights_scale", F32, c["weights_scale"]))
    tensors, strides = [], {}
    for layer, name, t, data, rows, cols in model["tensors"]:
        full = name if layer < 0 else f"blk.{layer}.{name}"
        full += "" if name.endswith("_bias") else ".weight"
        full = full.replace("_bias", ".bias")
        if name.endswith("_exps"):
            E = c["n_expert"]
            dims = [cols, rows // E, E]
            if prepared:
                strides[full] = (data.size // E + ALIGN + ALIGN - 1) // ALIGN * ALIGN
        elif rows == 1:
            dims = [cols]
        else:
            dims = [cols, rows]
        tensors.append((full, t, dims, np.ascontiguousarray(data)))
    write_gguf(path, meta, tensors, prepared=prepared, strides=strides)
