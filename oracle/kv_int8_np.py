"""CPU oracle of the opt-in INT8 prefix-KV decode attention.

TEST INFRASTRUCTURE ONLY.  Only ``tests/`` may import this module; the CUDA path in ``viktor_b200`` never calls
into it.

The reference has no int8 kernel.  Its design notes (analysis.md:95) propose the mode: the prefix KV is written
once, so it can be stored as int8 with per-channel scale factors, while the KV of generated tokens stays bf16.
This module restates the quantisation rule that the CUDA path defines for it, and the decode attention it
feeds (viktor/decode_attention.py:41-53 over a cache whose prefix is dequantized):

* per channel c (two KV heads x 64 = 128 channels) of one row: m_c = max over the prefix of |x[p, c]|,
  s_c = m_c / 127 and inv_c = 127 / m_c in fp32 (0 for an all-zero channel);
* stored byte u = clamp(rint(x * inv_c), -127, 127) + 128 (fp32 product, round half to even);
* the prefix value the attention sees is (u - 128) * s_c.

Parity unpinned against the reference (it ships no implementation of the mode): the bytes and scales are
checked bit-exactly against this restatement, the attention within a stated tolerance of its fp64 result, and
the quantisation error itself against the bf16 attention with a tolerance of its own.
"""

from __future__ import annotations

import numpy as np


def quantize_prefix(x: np.ndarray):
    """x [start, 128] float32 (bf16 values of one row, one layer) -> (bytes [start, 128] uint8, scale [128] f32)."""
    x = np.asarray(x, dtype=np.float32)
    m = np.abs(x).max(axis=0) if x.shape[0] else np.zeros(x.shape[1], np.float32)
    m = m.astype(np.float32)
    scale = (m / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(m > 0, np.float32(127) / m, np.float32(0)).astype(np.float32)
    q = np.clip(np.rint((x * inv).astype(np.float32)), -127, 127)
    return (q + 128).astype(np.uint8), scale


def dequantize(u: np.ndarray, scale: np.ndarray) -> np.ndarray:
    return (u.astype(np.float64) - 128.0) * scale.astype(np.float64)


def decode_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray) -> np.ndarray:
    """Single-query GQA attention in fp64: q [8, 64], k/v [L, 2, 64] -> [8, 64] (scale 1/8, head h reads KV head
    h // 4), viktor/decode_attention.py:41-53."""
    q = q.astype(np.float64)
    out = np.empty((8, 64))
    for h in range(8):
        kh, vh = k[:, h // 4].astype(np.float64), v[:, h // 4].astype(np.float64)
        s = kh @ q[h] / 8.0
        p = np.exp(s - s.max())
        out[h] = (p / p.sum()) @ vh
    return out


def decode_attention_i8(q, k, v, start):
    """q [8, 64]; k/v [L, 2, 64] (bf16 values) of one row: positions [0, start) quantized per channel as the
    CUDA path stores them, the rest kept exact.  Returns (out [8, 64] fp64, k bytes, k scale, v bytes, v scale)."""
    L = k.shape[0]
    k2 = np.asarray(k, np.float32).reshape(L, 128)
    v2 = np.asarray(v, np.float32).reshape(L, 128)
    ku, ks = quantize_prefix(k2[:start])
    vu, vs = quantize_prefix(v2[:start])
    kd = np.concatenate([dequantize(ku, ks), k2[start:].astype(np.float64)]).reshape(L, 2, 64)
    vd = np.concatenate([dequantize(vu, vs), v2[start:].astype(np.float64)]).reshape(L, 2, 64)
    return decode_attention(q, kd, vd), ku, ks, vu, vs
