"""GGML block formats: type table and a deterministic numpy quantizer.

The block layouts are GGUF's (Kestrel reads them in
crates/kestrel-engine/src/quant.rs:63-205 and sizes them in
crates/kestrel-gguf/src/types.rs:145-191). gguf-py can decode Q4_K/Q6_K but
cannot encode them, and llama-quantize is not available, so this module holds
this project's own quantizer. Its rules are simple and fully deterministic
(IEEE float32 arithmetic, round-half-to-even), and the CUDA quantizer
(`kc_quantize`) implements the same rules bit for bit, so weights generated on
the GPU for the benchmark equal the ones the tests generate here.

Parity never depends on quantizer quality: the GPU path and the CPU oracle
always consume the same bytes.
"""
from __future__ import annotations

import numpy as np

# ggml type ids (crates/kestrel-gguf/src/types.rs:48-86).
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 = 0, 1, 2, 3, 6, 7, 8
Q4_K, Q5_K, Q6_K, BF16 = 12, 13, 14, 30

NAMES = {F32: "F32", F16: "F16", Q4_0: "Q4_0", Q4_1: "Q4_1", Q5_0: "Q5_0", Q5_1: "Q5_1",
         Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", BF16: "BF16"}
BY_NAME = {v: k for k, v in NAMES.items()}

# (elements per block, bytes per block): types.rs:120-182.
BLOCK = {F32: (1, 4), F16: (1, 2), BF16: (1, 2), Q4_0: (32, 18), Q4_1: (32, 20), Q5_0: (32, 22),
         Q5_1: (32, 24), Q8_0: (32, 34), Q4_K: (256, 144), Q5_K: (256, 176), Q6_K: (256, 210)}


def bytes_for(t: int, n: int) -> int:
    """Bytes for `n` elements of type `t` (GgmlType::bytes_for, types.rs:185-191)."""
    be, bb = BLOCK[t]
    if n % be:
        raise ValueError(f"{NAMES[t]}: {n} elements is not a multiple of the block size {be}")
    return n // be * bb


def xorshift_bytes(n: int, seed: int) -> np.ndarray:
    """The reference tests' byte stream: xorshift32 (13, 17, 5), low byte of
    each state (qdot.rs:275-285, avx2.rs:172-182, avx2.rs:434-442)."""
    x = np.uint32(max(seed, 1))
    out = np.empty(n, dtype=np.uint8)
    # Vectorising a serial PRNG does not help; the test sizes are small.
    xs = int(x)
    for i in range(n):
        xs ^= (xs << 13) & 0xFFFFFFFF
        xs ^= xs >> 17
        xs ^= (xs << 5) & 0xFFFFFFFF
        out[i] = xs & 0xFF
    return out


def f16_bytes(v: float) -> bytes:
    return np.float16(v).tobytes()


def set_block_scales(raw: np.ndarray, t: int, value: float) -> np.ndarray:
    """Overwrite every block's f16 scale fields with `value`, as the reference
    tests do after drawing random bytes (qdot.rs:286-297, avx2.rs:199-208,
    avx2.rs:443-448)."""
    be, bb = BLOCK[t]
    offs = {Q8_0: [0], Q4_0: [0], Q5_0: [0], Q4_1: [0, 2], Q5_1: [0, 2], Q4_K: [0, 2],
            Q5_K: [0, 2], Q6_K: [208]}[t]
    blocks = raw.reshape(-1, bb).copy()
    h = np.frombuffer(f16_bytes(value), dtype=np.uint8)
    for o in offs:
        blocks[:, o:o + 2] = h
    return blocks.reshape(-1)


# ----------------------------------------------------------------------------
# Quantizer. All arithmetic in float32; round-half-to-even (np.rint).

def _f16_round(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).astype(np.float32)


def _safe_div(num: np.ndarray, den: np.ndarray) -> np.ndarray:
    """num / den (IEEE float32) where den > 0, else 0."""
    out = np.zeros(np.broadcast_shapes(num.shape, den.shape), np.float32)
    np.divide(num, den, out=out, where=den > 0)
    return out


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Q8_0: per 32, d = f16(amax/127), q = rint(x * (1/d)) clipped to +-127."""
    xb = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.abs(xb).max(axis=1)
    d16 = _f16_round(amax / np.float32(127))
    inv = _safe_div(np.ones_like(d16), d16)
    q = np.clip(np.rint(xb * inv[:, None]), -127, 127).astype(np.int8)
    out = np.empty((xb.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d16.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def quantize_q4_0(x: np.ndarray) -> np.ndarray:
    """Q4_0: per 32, d = f16(amax/7), q = rint(x/d)+8 clipped to 0..15."""
    xb = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    d16 = _f16_round(np.abs(xb).max(axis=1) / np.float32(7))
    q = np.clip(np.rint(_safe_div(xb, np.broadcast_to(d16[:, None], xb.shape))) + 8, 0, 15).astype(np.uint8)
    out = np.empty((xb.shape[0], 18), dtype=np.uint8)
    out[:, 0:2] = d16.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, :16] | (q[:, 16:] << 4)
    return out.reshape(-1)


def quantize_q4_k(x: np.ndarray) -> np.ndarray:
    """Q4_K: superblocks of 256 = 8 sub-blocks of 32 with 6-bit scale and min.

    Per sub-block j: lo_j = min(0, min x), scale_j = (max x - lo_j)/15,
    min_j = 0 - lo_j. Superblock d = f16(max scale_j / 63), dmin =
    f16(max min_j / 63); sc_j = rint(scale_j/d), m_j = rint(min_j/dmin) (0..63);
    q = rint((x + dmin*m_j) / (d*sc_j)) clipped to 0..15, so that the
    dequantised value is d*sc_j*q - dmin*m_j (quant.rs:138-155).
    """
    xb = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 8, 32)
    nb = xb.shape[0]
    lo = np.minimum(xb.min(axis=2), np.float32(0))
    hi = xb.max(axis=2)
    scale = ((hi - lo) / np.float32(15) + np.float32(0)).astype(np.float32)  # +0.0 for constant blocks
    mins = (np.float32(0) - lo).astype(np.float32)  # +0.0, never -0.0, for non-negative blocks
    d16 = _f16_round(scale.max(axis=1) / np.float32(63))
    dm16 = _f16_round(mins.max(axis=1) / np.float32(63))
    sc = np.clip(np.rint(_safe_div(scale, np.broadcast_to(d16[:, None], scale.shape))), 0, 63).astype(np.int32)
    mm = np.clip(np.rint(_safe_div(mins, np.broadcast_to(dm16[:, None], mins.shape))), 0, 63).astype(np.int32)
    D = (d16[:, None] * sc.astype(np.float32)).astype(np.float32)
    M = (dm16[:, None] * mm.astype(np.float32)).astype(np.float32)
    q = np.clip(np.rint(_safe_div(xb + M[:, :, None], np.broadcast_to(D[:, :, None], xb.shape))), 0, 15)
    q = q.astype(np.uint8)
    out = np.zeros((nb, 144), dtype=np.uint8)
    out[:, 0:2] = d16.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:4] = dm16.astype(np.float16).view(np.uint8).reshape(-1, 2)
    s = np.zeros((nb, 12), dtype=np.int32)
    # Inverse of scale_min_k4 (quant.rs:54-60).
    s[:, 0:4] = sc[:, 0:4] | ((sc[:, 4:8] >> 4) << 6)
    s[:, 4:8] = mm[:, 0:4] | ((mm[:, 4:8] >> 4) << 6)
    s[:, 8:12] = (sc[:, 4:8] & 0xF) | ((mm[:, 4:8] & 0xF) << 4)
    out[:, 4:16] = s.astype(np.uint8)
    # Element 64k+l -> low nibble of qs[32k+l]; 64k+32+l -> high nibble.
    qq = q.reshape(nb, 4, 2, 32)
    out[:, 16:144] = (qq[:, :, 0, :] | (qq[:, :, 1, :] << 4)).reshape(nb, 128)
    return out.reshape(-1)


def quantize_q6_k(x: np.ndarray) -> np.ndarray:
    """Q6_K: superblocks of 256 = 16 sub-blocks of 16 with an int8 scale.

    Per sub-block j: s_j = amax_j/31; d = f16(max s_j / 127); sc_j = rint(s_j/d)
    (0..127); q = rint(x/(d*sc_j)) clipped to -32..31, stored +32 as 6 bits so
    that the dequantised value is d*sc_j*(u-32) (quant.rs:180-201).
    """
    xb = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 16, 16)
    nb = xb.shape[0]
    s = (np.abs(xb).max(axis=2) / np.float32(31)).astype(np.float32)
    d16 = _f16_round(s.max(axis=1) / np.float32(127))
    sc = np.clip(np.rint(_safe_div(s, np.broadcast_to(d16[:, None], s.shape))), -128, 127).astype(np.int32)
    D = (d16[:, None] * sc.astype(np.float32)).astype(np.float32)
    q = np.clip(np.rint(_safe_div(xb, np.broadcast_to(D[:, :, None], xb.shape))), -32, 31).astype(np.int32) + 32
    q = q.reshape(nb, 2, 4, 32)  # [h][r][l]: element h*128 + 32r + l
    out = np.zeros((nb, 210), dtype=np.uint8)
    for h in range(2):
        q1, q2, q3, q4 = q[:, h, 0], q[:, h, 1], q[:, h, 2], q[:, h, 3]
        out[:, h * 64: h * 64 + 32] = ((q1 & 0xF) | ((q3 & 0xF) << 4)).astype(np.uint8)
        out[:, h * 64 + 32: h * 64 + 64] = ((q2 & 0xF) | ((q4 & 0xF) << 4)).astype(np.uint8)
        out[:, 128 + h * 32: 128 + h * 32 + 32] = (
            (q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)).astype(np.uint8)
    out[:, 192:208] = sc.astype(np.int8).view(np.uint8)
    out[:, 208:210] = d16.astype(np.float16).view(np.uint8).reshape(-1, 2)
    return out.reshape(-1)


QUANTIZERS = {Q8_0: quantize_q8_0, Q4_0: quantize_q4_0, Q4_K: quantize_q4_k, Q6_K: quantize_q6_k}


def quantize(t: int, x: np.ndarray) -> np.ndarray:
    """Quantize a float32 matrix `[rows, cols]` (cols contiguous) to type `t`.
    Returns the GGUF bytes `[rows, bytes_for(t, cols)]` as uint8."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.reshape(-1, x.shape[-1]).shape
    if t == F32:
        return x.view(np.uint8).reshape(rows, cols * 4)
    if t == F16:
        return x.astype(np.float16).view(np.uint8).reshape(rows, cols * 2)
    bytes_for(t, cols)
    return QUANTIZERS[t](x).reshape(rows, -1)
