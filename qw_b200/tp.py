"""Tensor-parallel partition of the 27B linear stack across P GPUs of one node.

The reference has no tensor parallelism (it is a single-device server); this
is the partition BASELINE asks for, Megatron style:

* column-parallel (no collective): q, k, v, gate, up and lm_head.  Each rank
  holds rows [r*N/P, (r+1)*N/P) of every fused plane (q|k|v and gate|up are
  sharded plane by plane, then re-fused per rank, so every rank holds N/P rows
  of each plane), with their scales and biases;
* row-parallel (fp32 allreduce): o and down.  Each rank holds input columns
  [r*K/P, (r+1)*K/P) of the packed weight, on group boundaries so that every
  quantization group (and its scale/bias) lies wholly in one shard; the rank's
  matmul returns fp32 partial sums that an allreduce adds before the single
  fp16 rounding.

Everything here is array slicing and works on numpy arrays or torch tensors.
"""
from __future__ import annotations

from typing import Callable, Dict, List, Sequence, Tuple

from . import synth

GROUP = synth.GROUP
WORDS_PER_GROUP = GROUP * synth.BITS // 32

# plane boundaries of the fused matrices (output features)
PLANES = {
    "qkv": (synth.Q_OUT, synth.KV_OUT, synth.KV_OUT),
    "gate_up": (synth.INTER, synth.INTER),
}


def split_even(n: int, parts: int, rank: int, align: int = 1) -> Tuple[int, int]:
    """[start, stop) of rank's share of n items, in multiples of `align`."""
    if n % align:
        raise ValueError(f"{n} is not a multiple of {align}")
    units = n // align
    if units % parts:
        raise ValueError(f"{n} does not split into {parts} shards of whole multiples of {align}")
    per = units // parts
    return rank * per * align, (rank + 1) * per * align


def column_shard_rows(name: str, N: int, P: int, rank: int) -> List[Tuple[int, int]]:
    """Row ranges of the full matrix that rank r holds, plane by plane."""
    planes = PLANES.get(name, (N,))
    assert sum(planes) == N
    out, base = [], 0
    for n in planes:
        a, b = split_even(n, P, rank)
        out.append((base + a, base + b))
        base += n
    return out


def row_shard_cols(K: int, P: int, rank: int) -> Tuple[int, int]:
    """Input-column range [k0, k1) of rank r; whole quantization groups."""
    return split_even(K, P, rank, align=GROUP)


def _cat(parts):
    if hasattr(parts[0], "new_empty"):  # torch
        import torch
        return torch.cat(parts, 0).contiguous()
    import numpy as np
    return np.ascontiguousarray(np.concatenate(parts, 0))


def shard_linear(lin: synth.Linear, wq, scales, biases, P: int, rank: int):
    """The rank's (wq, scales, biases) of a full quantized matrix."""
    if P == 1:
        return wq, scales, biases
    if lin.row_parallel:
        k0, k1 = row_shard_cols(lin.K, P, rank)
        w0, w1 = k0 * synth.BITS // 32, k1 * synth.BITS // 32
        g0, g1 = k0 // GROUP, k1 // GROUP
        return (_cat([wq[:, w0:w1]]), _cat([scales[:, g0:g1]]), _cat([biases[:, g0:g1]]))
    rows = column_shard_rows(lin.name, lin.N, P, rank)
    return (_cat([wq[a:b] for a, b in rows]), _cat([scales[a:b] for a, b in rows]),
            _cat([biases[a:b] for a, b in rows]))


def shard_shape(lin: synth.Linear, P: int) -> Tuple[int, int]:
    """(N, K) of one rank's shard."""
    if lin.row_parallel:
        return lin.N, lin.K // P
    return lin.N // P, lin.K


def local_input_cols(lin: synth.Linear, P: int, rank: int) -> Tuple[int, int]:
    """Columns of the full activation a row-parallel op consumes on this rank."""
    return row_shard_cols(lin.K, P, rank) if lin.row_parallel else (0, lin.K)


class LinearStack:
    """The decode linear stack on one rank: per layer qkv -> o -> gate_up ->
    down, then lm_head.  The stack keeps the data dependencies of a decoder
    layer without its non-linear parts (attention, norms, SwiGLU are outside
    this path): o consumes the q plane of the rank's qkv output, down consumes
    the gate plane of its gate_up output, and each layer's down output is the
    next layer's input.

    `matmul(x, (wq, s, b), out_f32)` runs one quantized matmul; `allreduce(t)`
    sums an fp32 tensor over ranks in place; `to_half(t)` rounds fp32 to fp16.
    """

    def __init__(self, layers: Sequence[Dict[str, tuple]], lm_head: tuple, P: int, rank: int,
                 matmul: Callable, allreduce: Callable, to_half: Callable):
        self.layers, self.lm_head = layers, lm_head
        self.P, self.rank = P, rank
        self.matmul, self.allreduce, self.to_half = matmul, allreduce, to_half
        self.lin = {l.name: l for l in synth.layer_linears()}

    def layer(self, h, w):
        P = self.P
        q_local = synth.Q_OUT // P
        inter_local = synth.INTER // P
        qkv = self.matmul(h, w["qkv"], False)
        attn = qkv[..., :q_local]
        if P == 1:
            o = self.matmul(_contig(attn), w["o"], False)
        else:
            o = self.to_half(self.allreduce(self.matmul(_contig(attn), w["o"], True)))
        gu = self.matmul(o, w["gate_up"], False)
        g = gu[..., :inter_local]
        if P == 1:
            return self.matmul(_contig(g), w["down"], False)
        return self.to_half(self.allreduce(self.matmul(_contig(g), w["down"], True)))

    def forward(self, h):
        for w in self.layers:
            h = self.layer(h, w)
        return self.matmul(h, self.lm_head, False)


def _contig(t):
    if hasattr(t, "is_contiguous"):
        return t if t.is_contiguous() else t.contiguous()
    import numpy as np
    return np.ascontiguousarray(t)
