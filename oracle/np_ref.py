"""Independent numpy restatement of the oracle (TEST INFRASTRUCTURE).

Written separately from qw_oracle.c so the two can check each other:
unpacking uses vectorised shifts instead of per-element loops, dequantize is
evaluated with numpy's own float16 arithmetic, and the matmul accumulates in
float64.  Same semantics and citations as qw_oracle.h.
"""
from __future__ import annotations

import numpy as np


def unpack(wq: np.ndarray, bits: int = 4) -> np.ndarray:
    """uint32 [N, K*bits/32] -> uint8 codes [N, K], lowest bits first."""
    pf = 32 // bits
    shifts = (np.arange(pf, dtype=np.uint32) * bits)[None, None, :]
    codes = (wq[:, :, None] >> shifts) & np.uint32((1 << bits) - 1)
    return codes.reshape(wq.shape[0], -1).astype(np.uint8)


def pack(codes: np.ndarray, bits: int = 4) -> np.ndarray:
    pf = 32 // bits
    N, K = codes.shape
    c = codes.astype(np.uint32).reshape(N, K // pf, pf)
    shifts = (np.arange(pf, dtype=np.uint32) * bits)[None, None, :]
    return np.bitwise_or.reduce(c << shifts, axis=2).astype(np.uint32)


def dequantize(wq, scales, biases, group_size=64, bits=4, rounding="twice"):
    q = unpack(wq, bits).astype(np.float16)
    s = np.repeat(scales.astype(np.float16), group_size, axis=1)
    b = np.repeat(biases.astype(np.float16), group_size, axis=1)
    if rounding == "twice":
        # numpy float16 ops round each result to nearest-even binary16
        return (s * q) + b
    # rounded once: exact in float64, then a single rounding to binary16
    exact = s.astype(np.float64) * q.astype(np.float64) + b.astype(np.float64)
    return exact.astype(np.float16)


def quantized_matmul(x, wq, scales, biases, group_size=64, bits=4):
    """float64-accumulated x . dequant(w)^T with the fp32-formed weight; returns float64."""
    q = unpack(wq, bits).astype(np.float32)
    s = np.repeat(scales.astype(np.float32), group_size, axis=1)
    b = np.repeat(biases.astype(np.float32), group_size, axis=1)
    w = (s * q) + b  # float32, like the oracle
    return x.astype(np.float64) @ w.astype(np.float64).T


def quantize(w, group_size=64, bits=4):
    """Vectorised restatement of qwo_quantize (float32 arithmetic throughout)."""
    w = np.asarray(w, dtype=np.float16)
    N, K = w.shape
    nb = np.float32((1 << bits) - 1)
    g = w.astype(np.float32).reshape(N, K // group_size, group_size)
    mn = g.min(axis=2)
    mx = g.max(axis=2)
    scale = (mx - mn) / nb
    scale = np.where(scale >= np.float32(1e-7), scale, np.float32(1e-7)).astype(np.float32)
    sh = scale.astype(np.float16)
    bh = mn.astype(np.float16)
    r = np.rint((g - bh.astype(np.float32)[..., None]) / sh.astype(np.float32)[..., None])
    codes = np.clip(r, 0, nb).astype(np.uint8).reshape(N, K)
    return pack(codes, bits), sh, bh
