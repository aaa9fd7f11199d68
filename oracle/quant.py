"""Groupwise expert-weight quantization, restated in numpy (TEST INFRASTRUCTURE ONLY).

The reference engine lists "Int8 and int4 groupwise expert weights" on its
roadmap (moe-inference-engine.md:36) and ships no code for it, so there is no
reference output to pin against: parity for this path is UNPINNED to the
reference.  This file restates the published method the product implements --
round-to-nearest symmetric absmax quantization in groups along the reduction
dimension of each row -- independently of torch, and the tests check the
product's quantizer against it bit for bit, the kernels against the MoE oracle
(``moe_decode_stacked``) run on the dequantized weights.

Per group of ``group`` consecutive elements of a row (fp32 arithmetic):
    scale = max_i |w_i| / qmax          (qmax = 127 for 8 bits, 7 for 4 bits)
    q_i   = clip(round_half_even(w_i / scale), -qmax, qmax)   (0 if scale == 0)
    w_i  ~ scale * q_i
4-bit values are stored two per byte, the even element in the low nibble, as
4-bit two's complement.
"""

from __future__ import annotations

import numpy as np


def quantize(w: np.ndarray, bits: int, group: int):
    """w float32 [E, R, C] -> (q int8 [E, R, C], scale float32 [E, R, C // group])."""
    if bits not in (8, 4):
        raise ValueError(bits)
    w = np.asarray(w, dtype=np.float32)
    E, R, C = w.shape
    qmax = np.float32(127 if bits == 8 else 7)
    g = w.reshape(E, R, C // group, group)
    scale = (np.abs(g).max(axis=-1) / qmax).astype(np.float32)
    safe = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(g / safe[..., None]), -qmax, qmax).astype(np.int8)
    return q.reshape(E, R, C), scale


def pack4(q: np.ndarray) -> np.ndarray:
    """int8 values in [-8, 7], [..., C] -> uint8 [..., C // 2] (even element low)."""
    u = (q.astype(np.int16) & 0xF).astype(np.uint8)
    return (u[..., 0::2] | (u[..., 1::2] << 4)).astype(np.uint8)


def unpack4(p: np.ndarray) -> np.ndarray:
    lo = (p & 0xF).astype(np.int16)
    hi = ((p >> 4) & 0xF).astype(np.int16)
    lo = np.where(lo >= 8, lo - 16, lo)
    hi = np.where(hi >= 8, hi - 16, hi)
    return np.stack((lo, hi), axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 2).astype(np.int8)


def dequantize(q: np.ndarray, scale: np.ndarray, group: int) -> np.ndarray:
    E, R, C = q.shape
    return (q.astype(np.float32).reshape(E, R, C // group, group) * scale[..., None]).reshape(E, R, C)
