"""CPU oracle for the affine group-quantized matmul (TEST INFRASTRUCTURE).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
(``cpu_baseline`` and ``--impl reference``) may import this package.  The
product library never calls it: it is the checker, not the thing measured.

The arithmetic lives in ``qw_oracle.c`` (see its header for the reference
citations).  ``np_ref`` holds an independent float64 numpy restatement used to
cross-check the C code.

Parity status: unpinned by the reference.  cr0sh/qw has no golden vectors for
this path and its MLX dependency cannot be built in this environment; the
oracle is pinned instead by hand-derived known answers, by the reference's own
layout-commutation test (crates/mlxcel-core/src/ffi_tests.rs:3792-3850) and by
the committed fixtures under tests/golden/.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libqworacle.so")
_lib = None

ROUND_TWICE = 0
ROUND_ONCE = 1


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        i32 = ctypes.c_int
        L.qwo_quantize.argtypes = [p, i64, i64, i32, i32, p, p, p]
        L.qwo_dequantize.argtypes = [p, p, p, i64, i64, i32, i32, i32, p]
        L.qwo_quantized_matmul.argtypes = [p, p, p, p, i64, i64, i64, i32, i32, p, p, i32]
        L.qwo_dequantize_f32.argtypes = [p, p, p, i64, i64, i32, i32, i32, p]
        L.qwo_matmul_f16w.argtypes = [p, p, i64, i64, i64, p, p, i32]
        L.qwo_f32_to_f16.argtypes = [ctypes.c_float]
        L.qwo_f32_to_f16.restype = ctypes.c_uint16
        L.qwo_f64_to_f16.argtypes = [ctypes.c_double]
        L.qwo_f64_to_f16.restype = ctypes.c_uint16
        L.qwo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.qwo_f16_to_f32.restype = ctypes.c_float
        L.qwo_max_threads.restype = i32
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def _check(rc: int, what: str):
    if rc != 0:
        raise ValueError(f"oracle {what} rejected its arguments (status {rc})")


def quantize(w: np.ndarray, group_size: int = 64, bits: int = 4):
    """Affine-quantize fp16 w [N, K] -> (wq uint32 [N, K*bits/32], scales, biases fp16 [N, K/gs])."""
    w = np.ascontiguousarray(w, dtype=np.float16)
    N, K = w.shape
    wq = np.zeros((N, K * bits // 32), dtype=np.uint32)
    s = np.zeros((N, K // group_size), dtype=np.float16)
    b = np.zeros((N, K // group_size), dtype=np.float16)
    _check(lib().qwo_quantize(_ptr(w), N, K, group_size, bits, _ptr(wq), _ptr(s), _ptr(b)), "quantize")
    return wq, s, b


def dequantize(wq, scales, biases, group_size: int = 64, bits: int = 4, rounding: int = ROUND_TWICE):
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    biases = np.ascontiguousarray(biases, dtype=np.float16)
    N = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    out = np.zeros((N, K), dtype=np.float16)
    _check(lib().qwo_dequantize(_ptr(wq), _ptr(scales), _ptr(biases), N, K, group_size, bits,
                                rounding, _ptr(out)), "dequantize")
    return out


def dequantize_f32(wq, scales, biases, group_size: int = 64, bits: int = 4, rounding: int = ROUND_TWICE):
    """dequantize for float32 scales and biases -> float32 [N, K]: ROUND_TWICE
    forms fp32(fp32(s*q) + b), ROUND_ONCE fmaf(s, q, b).  MLX returns the
    scales' dtype, so the reference's f32-scale layout test
    (crates/mlxcel-core/src/ffi_tests.rs:3792-3850) dequantizes to float32."""
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    biases = np.ascontiguousarray(biases, dtype=np.float32)
    N = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    out = np.zeros((N, K), dtype=np.float32)
    _check(lib().qwo_dequantize_f32(_ptr(wq), _ptr(scales), _ptr(biases), N, K, group_size, bits, rounding,
                                    _ptr(out)), "dequantize_f32")
    return out


def matmul_f16w(x, w16, nthreads: int = 0, want_f32: bool = False):
    """y = x . w16^T for fp16 weights [N, K]: products and sums in float32,
    ascending k, one rounding to fp16 at the end."""
    x = np.ascontiguousarray(x, dtype=np.float16)
    lead, K = x.shape[:-1], x.shape[-1]
    x2 = x.reshape(-1, K)
    w16 = np.ascontiguousarray(w16, dtype=np.float16)
    M, N = x2.shape[0], w16.shape[0]
    if w16.shape[1] != K:
        raise ValueError("w's K does not match x's")
    y = np.zeros((M, N), dtype=np.float16)
    y32 = np.zeros((M, N), dtype=np.float32) if want_f32 else None
    _check(lib().qwo_matmul_f16w(_ptr(x2), _ptr(w16), M, N, K, _ptr(y), _ptr(y32) if y32 is not None else None,
                                 nthreads), "matmul_f16w")
    y = y.reshape(*lead, N)
    return (y, y32.reshape(*lead, N)) if want_f32 else y


def quantized_matmul_f16acc(x, wq, scales, biases, group_size: int = 64, bits: int = 4):
    """The matmul evaluated wholly in fp16, one rounded operation at a time:
    w = dequantize(..., ROUND_TWICE), then acc = fp16(acc + fp16(x[k] * w[k]))
    in ascending k.  The reading of "every op in the output dtype" carried
    through the accumulation; used to bound how far such an evaluation lies
    from the float32-accumulated results (float32 arithmetic rounded to fp16
    is the correctly rounded fp16 result for one product or one sum of fp16
    operands)."""
    w = dequantize(wq, scales, biases, group_size=group_size, bits=bits).astype(np.float32)
    x = np.ascontiguousarray(x, dtype=np.float16).astype(np.float32)
    x2 = x.reshape(-1, x.shape[-1])
    acc = np.zeros((x2.shape[0], w.shape[0]), dtype=np.float16)
    for k in range(w.shape[1]):
        p = (x2[:, k:k + 1] * w[None, :, k]).astype(np.float16)
        acc = (acc.astype(np.float32) + p.astype(np.float32)).astype(np.float16)
    return acc.reshape(*x.shape[:-1], w.shape[0])


def quantized_matmul(x, wq, scales, biases, group_size: int = 64, bits: int = 4,
                     nthreads: int = 0, want_f32: bool = False, weights: str = "f32"):
    """y = x . dequantize(w)^T with fp32 accumulation; x fp16 [..., K].

    weights="f32" forms each weight as s*q + b in float32 (two rounded fp32
    ops); weights="f16" multiplies the fp16 ROUND_TWICE dequantized weights
    (the `dequantize` output) instead.  Both accumulate in float32 in
    ascending k."""
    if weights == "f16":
        return matmul_f16w(x, dequantize(wq, scales, biases, group_size=group_size, bits=bits),
                           nthreads=nthreads, want_f32=want_f32)
    if weights != "f32":
        raise ValueError(f"weights must be 'f32' or 'f16', got {weights!r}")
    x = np.ascontiguousarray(x, dtype=np.float16)
    lead = x.shape[:-1]
    K = x.shape[-1]
    x2 = x.reshape(-1, K)
    M = x2.shape[0]
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.float16)
    biases = np.ascontiguousarray(biases, dtype=np.float16)
    N = wq.shape[0]
    if wq.shape[1] * 32 // bits != K:
        raise ValueError("packed width does not match x's K")
    y = np.zeros((M, N), dtype=np.float16)
    y32 = np.zeros((M, N), dtype=np.float32) if want_f32 else None
    _check(lib().qwo_quantized_matmul(_ptr(x2), _ptr(wq), _ptr(scales), _ptr(biases), M, N, K,
                                      group_size, bits, _ptr(y),
                                      _ptr(y32) if y32 is not None else None, nthreads),
           "quantized_matmul")
    y = y.reshape(*lead, N)
    if want_f32:
        return y, y32.reshape(*lead, N)
    return y


def swiglu(gate, up):
    """silu(gate) * up on fp16 arrays, rounded to fp16 after every op: the
    reference's activation (mlx_cxx_bridge.cpp:1205-1216, silu_gate =
    gate * sigmoid(gate); out = silu_gate * x) evaluated on its fp16 matmul
    outputs, each elementwise op producing an fp16 array.  sigmoid is formed
    in float32 and rounded once."""
    g = np.asarray(gate, dtype=np.float16).astype(np.float32)
    u = np.asarray(up, dtype=np.float16).astype(np.float32)
    with np.errstate(over="ignore"):
        sig = (np.float32(1.0) / (np.float32(1.0) + np.exp(-g))).astype(np.float16).astype(np.float32)
    silu = (g * sig).astype(np.float16).astype(np.float32)
    return (silu * u).astype(np.float16)


def quantized_matmul_swiglu(x, gate, up, group_size: int = 64, bits: int = 4, nthreads: int = 0):
    """silu(x . gate^T) * (x . up^T) with gate/up = (wq, scales, biases):
    Mlp::forward_hidden (crates/runtime/src/qwen3_next.rs:463-487) as two
    quantized matmuls (fp16 outputs) and the activation above."""
    g = quantized_matmul(x, *gate, group_size=group_size, bits=bits, nthreads=nthreads)
    u = quantized_matmul(x, *up, group_size=group_size, bits=bits, nthreads=nthreads)
    return swiglu(g, u)


def topk(logits, k: int):
    """(indices int64 [..., k], values fp16 [..., k]): the k largest fp16
    logits of each row, descending, lower index first among equal values --
    one outcome of argpartition(logits, -k) + take_along_axis as
    top_k_candidate_logits uses them (crates/runtime/src/qwen3_5_dflash.rs:
    1236-1266).  Values compare by their order-preserving fp16 key (-0 below
    +0; NaN by bit pattern).  Requires 1 <= k < N (qwen3_5_dflash.rs:1248-1253)."""
    a = np.ascontiguousarray(logits, dtype=np.float16)
    N = a.shape[-1]
    if not 1 <= k < N:
        raise ValueError(f"k={k} must be in 1..{N - 1}")
    rows = a.reshape(-1, N)
    b = rows.view(np.uint16).astype(np.uint32)
    key = np.where(b & 0x8000, (~b) & 0xFFFF, b | 0x8000)
    idx = np.empty((rows.shape[0], k), dtype=np.int64)
    for m in range(rows.shape[0]):
        order = np.lexsort((np.arange(N), -key[m].astype(np.int64)))  # key descending, then index
        idx[m] = order[:k]
    vals = np.take_along_axis(rows, idx, axis=1)
    return idx.reshape(*a.shape[:-1], k), vals.reshape(*a.shape[:-1], k)


def max_threads() -> int:
    return int(lib().qwo_max_threads())
