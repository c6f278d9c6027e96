"""Seeded synthetic inputs with the shapes of the BASELINE configurations.

No dataset is involved: x ~ N(0, 1) and W ~ N(0, 0.02) in fp16, W then
affine-quantized with group 64 / 4 bits.  Seeds are (seed, layer, tensor id)
sub-streams so that any single layer can be regenerated on its own.

The 27B linear stack runs the reference's load-time fusions
(q|k|v planes concatenated along N, crates/mlxcel-core/src/layers.rs:2467-2850;
gate|up, crates/runtime/src/qwen3_next.rs:406-447), so each layer is four
quantized matmuls: qkv 5120->8192, o 6144->5120, gate_up 5120->34816,
down 17408->5120; the stack ends with lm_head 5120->151936.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import numpy as np

HIDDEN = 5120
Q_OUT = 6144
KV_OUT = 1024
INTER = 17408
VOCAB = 151936
LAYERS = 64
GROUP = 64
BITS = 4


@dataclass(frozen=True)
class Linear:
    name: str
    N: int  # out features
    K: int  # in features
    tid: int  # tensor id for seeding
    row_parallel: bool  # tensor-parallel split along K (True) or N (False)


def layer_linears() -> List[Linear]:
    return [
        Linear("qkv", Q_OUT + 2 * KV_OUT, HIDDEN, 0, False),
        Linear("o", HIDDEN, Q_OUT, 1, True),
        Linear("gate_up", 2 * INTER, HIDDEN, 2, False),
        Linear("down", HIDDEN, INTER, 3, True),
    ]


LM_HEAD = Linear("lm_head", VOCAB, HIDDEN, 9, False)


def quant_bytes(N: int, K: int) -> int:
    """Packed weights + fp16 scales + fp16 biases."""
    return N * K // 2 + 2 * 2 * N * (K // GROUP)


def algorithmic_bytes(M: int, N: int, K: int) -> int:
    """Bytes one quantized matmul must move: weights, scales, biases, x and y."""
    return quant_bytes(N, K) + 2 * M * K + 2 * M * N


def stack_bytes(M: int, layers: int = LAYERS, lm_head: bool = True) -> int:
    b = layers * sum(algorithmic_bytes(M, l.N, l.K) for l in layer_linears())
    if lm_head:
        b += algorithmic_bytes(M, LM_HEAD.N, LM_HEAD.K)
    return b


def stack_flops(M: int, layers: int = LAYERS, lm_head: bool = True) -> int:
    f = layers * sum(2 * M * l.N * l.K for l in layer_linears())
    if lm_head:
        f += 2 * M * LM_HEAD.N * LM_HEAD.K
    return f


def rng(seed: int, layer: int, tid: int) -> np.random.Generator:
    return np.random.default_rng([seed, layer, tid])


def weight_fp16(N: int, K: int, seed: int = 0, layer: int = 0, tid: int = 0, std: float = 0.02) -> np.ndarray:
    """N x K fp16 ~ N(0, std).  std = K ** -0.5 keeps activations at unit
    scale through a stack without norms (the SwiGLU stacks of the tests)."""
    g = rng(seed, layer, tid)
    return (g.standard_normal((N, K), dtype=np.float32) * np.float32(std)).astype(np.float16)


def activations(M: int, K: int, seed: int = 0, tid: int = 99) -> np.ndarray:
    g = rng(seed, 1000, tid)
    return g.standard_normal((M, K), dtype=np.float32).astype(np.float16)
