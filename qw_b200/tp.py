"""Tensor-parallel partition of the 27B linear stack across P GPUs of one node.

The reference has no tensor parallelism (it is a single-device server); this
is the partition BASELINE asks for, Megatron style:

* column-parallel (no collective): q, k, v, gate, up and lm_head.  Each rank
  holds rows [r*N/P, (r+1)*N/P) of every plane of a fused matrix (q|k|v and
  gate|up are sharded plane by plane, then re-fused per rank), with their
  scales and biases;
* row-parallel (fp32 sum over ranks): o and down.  Each rank holds input
  columns [r*K/P, (r+1)*K/P) of the packed weight, on group boundaries so that
  every quantization group (and its scale/bias) lies wholly in one shard; the
  ranks' fp32 products are added before the single fp16 rounding, inside the
  decode kernel (PeerAllreduce.matmul, the library's qw_allreduce_matmul), by
  the library's allreduce kernel after a matmul into fp32 (PeerAllreduce), or
  by NCCL.

Everything here is slicing and works on numpy arrays or torch tensors.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Sequence, Tuple

from . import synth

GROUP = synth.GROUP


@dataclass(frozen=True)
class StackDims:
    """Widths of one decoder layer's linears (defaults: the BASELINE 27B stack)."""
    hidden: int = synth.HIDDEN
    q_out: int = synth.Q_OUT
    kv_out: int = synth.KV_OUT
    inter: int = synth.INTER
    vocab: int = synth.VOCAB

    def linears(self) -> List[synth.Linear]:
        return [
            synth.Linear("qkv", self.q_out + 2 * self.kv_out, self.hidden, 0, False),
            synth.Linear("o", self.hidden, self.q_out, 1, True),
            synth.Linear("gate_up", 2 * self.inter, self.hidden, 2, False),
            synth.Linear("down", self.hidden, self.inter, 3, True),
        ]

    def lm_head(self) -> synth.Linear:
        return synth.Linear("lm_head", self.vocab, self.hidden, 9, False)

    def planes(self, name: str, N: int) -> Tuple[int, ...]:
        if name == "qkv":
            return (self.q_out, self.kv_out, self.kv_out)
        if name == "gate_up":
            return (self.inter, self.inter)
        return (N,)


BASELINE = StackDims()


def split_even(n: int, parts: int, rank: int, align: int = 1) -> Tuple[int, int]:
    """[start, stop) of rank's share of n items, in multiples of `align`."""
    if n % align:
        raise ValueError(f"{n} is not a multiple of {align}")
    units = n // align
    if units % parts:
        raise ValueError(f"{n} does not split into {parts} shards of whole multiples of {align}")
    per = units // parts
    return rank * per * align, (rank + 1) * per * align


def column_shard_rows(lin: synth.Linear, P: int, rank: int, dims: StackDims = BASELINE) -> List[Tuple[int, int]]:
    """Row ranges of the full matrix that rank r holds, plane by plane."""
    planes = dims.planes(lin.name, lin.N)
    assert sum(planes) == lin.N
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


def shard_linear(lin: synth.Linear, wq, scales, biases, P: int, rank: int, dims: StackDims = BASELINE):
    """The rank's (wq, scales, biases) of a full quantized matrix."""
    if P == 1:
        return wq, scales, biases
    if lin.row_parallel:
        k0, k1 = row_shard_cols(lin.K, P, rank)
        w0, w1 = k0 * synth.BITS // 32, k1 * synth.BITS // 32
        g0, g1 = k0 // GROUP, k1 // GROUP
        return (_cat([wq[:, w0:w1]]), _cat([scales[:, g0:g1]]), _cat([biases[:, g0:g1]]))
    rows = column_shard_rows(lin, P, rank, dims)
    return (_cat([wq[a:b] for a, b in rows]), _cat([scales[a:b] for a, b in rows]),
            _cat([biases[a:b] for a, b in rows]))


def shard_shape(lin: synth.Linear, P: int) -> Tuple[int, int]:
    """(N, K) of one rank's shard."""
    if lin.row_parallel:
        return lin.N, lin.K // P
    return lin.N // P, lin.K


class LinearStack:
    """The decode linear stack on one rank: per layer qkv -> o -> gate_up ->
    down, then lm_head.  The stack keeps the data dependencies of a decoder
    layer without attention and norms: o consumes the rank's q plane of its
    qkv output, down consumes silu(gate) * up of the rank's gate and up planes
    (or, without a `swiglu` callable, the gate plane as it is), and each
    layer's down output is the next layer's input.

    `matmul(x, (wq, s, b), out_f32)` runs one quantized matmul; `allreduce(t)`
    sums an fp32 array over ranks and returns it; `to_half(t)` rounds fp32 to
    fp16; `swiglu(x, (wq, s, b))` (optional) returns silu(gate) * up of the
    rank's gate_up shard, whose first half of rows is its gate plane and
    second half the matching up rows, so the activation needs no exchange
    between ranks; `rowpar(x, (wq, s, b))` (optional) runs a row-parallel
    projection with its sum over ranks in one call and returns fp16 (the
    library's qw_allreduce_matmul) in place of matmul, allreduce and to_half.
    Row-parallel shards need every rank to run the same sequence of
    collectives, which this fixed order guarantees.
    """

    def __init__(self, layers: Sequence[Dict[str, tuple]], lm_head: tuple, P: int, rank: int,
                 matmul: Callable, allreduce: Callable, to_half: Callable, dims: StackDims = BASELINE,
                 swiglu: Callable = None, rowpar: Callable = None):
        self.layers, self.lm_head = layers, lm_head
        self.P, self.rank, self.dims = P, rank, dims
        self.matmul, self.allreduce, self.to_half = matmul, allreduce, to_half
        self.swiglu, self.rowpar = swiglu, rowpar

    def _rowpar(self, x, w):
        if self.P == 1:
            return self.matmul(x, w, False)
        if self.rowpar is not None:
            return self.rowpar(x, w)
        return self.to_half(self.allreduce(self.matmul(x, w, True)))

    def layer(self, h, w):
        q_local = self.dims.q_out // self.P
        inter_local = self.dims.inter // self.P
        qkv = self.matmul(h, w["qkv"], False)
        o = self._rowpar(_contig(qkv[..., :q_local]), w["o"])
        if self.swiglu is not None:
            return self._rowpar(self.swiglu(o, w["gate_up"]), w["down"])
        gu = self.matmul(o, w["gate_up"], False)
        return self._rowpar(_contig(gu[..., :inter_local]), w["down"])

    def forward(self, h):
        for w in self.layers:
            h = self.layer(h, w)
        return self.matmul(h, self.lm_head, False)


# ---------------------------------------------------------------- greedy token
# A row's best logit as one integer key: the fp16 value made order-preserving
# (its float32 bits, sign-folded) above, 2^32 - 1 - (global index) below, so
# the largest key is the largest logit and, among equal logits, the lowest
# global index -- the rule of argmax_last_axis (lib.rs:2055) over the whole
# vocabulary.  The library's decode-kernel epilogue and qw_allreduce_argmax
# use the same key; the helpers below are its host-side statement (for the
# NCCL exchange and the CPU tests).
_SIGN64 = 1 << 63


def greedy_keys(logits, index_base: int = 0):
    """uint64 key of the best logit of each row of fp16 logits [..., N]
    whose first column is vocabulary row index_base (numpy)."""
    import numpy as np
    a = np.asarray(logits, dtype=np.float16)
    N = a.shape[-1]
    b = a.reshape(-1, N).astype(np.float32).view(np.uint32).astype(np.uint64)
    ordered = np.where(b & 0x80000000, (~b) & 0xFFFFFFFF, b | 0x80000000)
    low = np.uint64(0xFFFFFFFF) - (np.uint64(index_base) + np.arange(N, dtype=np.uint64))
    return ((ordered << np.uint64(32)) | low[None, :]).max(axis=1).reshape(a.shape[:-1])


def key_index(keys):
    """Global index held in greedy keys (numpy uint64 or torch int64 of
    signed_keys)."""
    if hasattr(keys, "new_empty"):  # torch: signed keys
        return (0xFFFFFFFF - (keys & 0xFFFFFFFF)).to(keys.dtype)
    import numpy as np
    return (np.uint64(0xFFFFFFFF) - (np.asarray(keys, np.uint64) & np.uint64(0xFFFFFFFF))).astype(np.int64)


def signed_keys(keys):
    """uint64 keys as int64 that compare the same way (for an int64 MAX
    all-reduce, which NCCL and gloo provide)."""
    import numpy as np
    return (np.asarray(keys, np.uint64) ^ np.uint64(_SIGN64)).view(np.int64)


def greedy_keys_torch(logits, index_base: int = 0):
    """signed_keys(greedy_keys(...)) of torch fp16 logits [..., N], on their device."""
    import torch
    N = logits.shape[-1]
    b = logits.reshape(-1, N).float().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    ordered = torch.where((b & 0x80000000) != 0, (~b) & 0xFFFFFFFF, b | 0x80000000)
    low = 0xFFFFFFFF - (index_base + torch.arange(N, device=logits.device, dtype=torch.int64))
    # bit 63 flipped before the signed max: signed order = the keys' unsigned order
    k = (((ordered << 32) | low) ^ (-_SIGN64)).max(dim=1).values
    return k.reshape(logits.shape[:-1])


def exchange_greedy_keys(keys_signed, group=None):
    """The global greedy token of each row from every rank's signed keys: an
    int64 MAX all-reduce over `group` (torch.distributed, any backend), then
    the index."""
    import torch.distributed as dist
    dist.all_reduce(keys_signed, op=dist.ReduceOp.MAX, group=group)
    return key_index(keys_signed)


def gate_up_halves(w):
    """(gate, up) triples of a rank's gate_up shard (rows: gate plane, then up)."""
    n = w[0].shape[0] // 2
    return tuple(t[:n] for t in w), tuple(t[n:] for t in w)


def _contig(t):
    if hasattr(t, "is_contiguous"):
        return t if t.is_contiguous() else t.contiguous()
    import numpy as np
    return np.ascontiguousarray(t)


def gather_columns(shards: Sequence, lin: synth.Linear, dims: StackDims = BASELINE):
    """Reassemble a column-parallel output [.., N] from every rank's [.., N/P]
    (plane by plane), e.g. the full logits from the vocab shards."""
    import numpy as np
    P = len(shards)
    planes = dims.planes(lin.name, lin.N)
    out, base_local = [], 0
    for n in planes:
        per = n // P
        out.extend(np.asarray(s)[..., base_local:base_local + per] for s in shards)
        base_local += per
    return np.concatenate(out, axis=-1)


class PeerAllreduce:
    """fp32 partial sums of a row-parallel projection summed over the ranks of
    a torch.distributed group (one process per GPU of one node) by the
    library's one-shot NVLink kernel (qw_allreduce_sum), with the fp16
    rounding fused: the exchange step of the tensor-parallel stack in place
    of ncclAllReduce + a cast.  The IPC handles travel over `group` (any
    backend) once, at construction."""

    def __init__(self, max_elems: int, group=None):
        import ctypes

        import torch
        import torch.distributed as dist

        from . import _lib
        self._lib = _lib
        L = _lib.load()
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        comm = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(_lib.QW_IPC_HANDLE_BYTES)
        _lib.check(L.qw_allreduce_init(world, rank, int(max_elems), ctypes.byref(comm), handle))
        self._comm = comm
        mine = list(handle.raw)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine, group=group)
        blob = bytes(b for h in gathered for b in h)
        _lib.check(L.qw_allreduce_connect(self._comm, blob))
        dist.barrier(group=group)
        self.world, self.rank, self.max_elems = world, rank, int(max_elems)
        self._group = group
        self._device = torch.cuda.current_device()

    def argmax(self, x, w, index_base: int, idx=None, logits=None, group_size: int = 64, bits: int = 4,
               mode: str = "affine"):
        """Global greedy token of each row of x over the ranks' vocabulary
        shards (qw_allreduce_argmax): this rank's shard w = (wq, scales,
        biases) holds vocabulary rows [index_base, index_base + N).  Returns
        int64 [M] indices, the same on every rank."""
        import torch

        from .ops import _arr, _mode, _stream
        M = x.numel() // x.shape[-1]
        if idx is None:
            idx = torch.empty(M, dtype=torch.int32, device=x.device)
        self._lib.check(self._lib.load().qw_allreduce_argmax(
            self._comm, _arr(x), _arr(w[0]), _arr(w[1]), _arr(w[2]), group_size, bits, _mode(mode),
            int(index_base), _arr(logits), _arr(idx), _stream(x)))
        return idx

    def matmul(self, x, w, out, group_size: int = 64, bits: int = 4, mode: str = "affine"):
        """Row-parallel projection (qw_allreduce_matmul): out (fp16 or fp32
        [M, N]) = the sum over ranks of each rank's x @ dequantize(w).T over
        its K-slice, summed in rank order and rounded once.  For M <= 16 the
        exchange runs in the decode kernel's epilogue (one launch)."""
        from .ops import _arr, _mode, _stream
        self._lib.check(self._lib.load().qw_allreduce_matmul(
            self._comm, _arr(x), _arr(w[0]), _arr(w[1]), _arr(w[2]), group_size, bits, _mode(mode), _arr(out),
            _stream(x)))
        return out

    def __call__(self, partial, out):
        """out (fp16 or fp32) = sum over ranks of partial (fp32, same numel)."""
        from .ops import _arr, _stream
        self._lib.check(self._lib.load().qw_allreduce_sum(self._comm, _arr(partial), _arr(out), _stream(partial)))
        return out

    def close(self, barrier: bool = True):
        """Free this rank's buffer and its mappings of the peers' buffers.
        Peers store into this rank's buffer during their calls (a call that
        gave up on a missing peer may store late), so no rank may free its
        buffer before every rank's calls have ended.  With barrier=True this
        waits for the device's work and then for every rank of the group, so
        every rank must call close; pass False only when the caller has done
        both itself."""
        if self._comm:
            if barrier:
                import torch
                import torch.distributed as dist
                torch.cuda.synchronize(self._device)
                dist.barrier(group=self._group)
            self._lib.load().qw_allreduce_destroy(self._comm)
            self._comm = None
