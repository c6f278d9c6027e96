"""Host-side mirror of mlxcel-core's quantized-linear operator surface.

Each function keeps the name, argument meaning and error behaviour of the
cxx bridge function it stands in for (crates/mlxcel-core/src/lib.rs), with
torch CUDA tensors in place of MlxArray and a raise in place of the bridge's
uncatchable abort.  The work happens in libqwqmm.so through its C ABI; torch
supplies device memory and the current stream only.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib

_DT = {
    torch.float16: _lib.QW_F16,
    torch.bfloat16: _lib.QW_BF16,
    torch.float32: _lib.QW_F32,
    torch.int32: _lib.QW_U32,   # MLX's uint32 packing, viewed as int32 by torch
    torch.uint32: _lib.QW_U32,
}


# Descriptors by (address, dtype, shape, strides): a descriptor holds nothing
# else, so equal keys share one, and a decode loop that calls with the same
# weights and buffers every step builds each once.  The library reads a
# descriptor only during the call.
_DESC_CACHE: dict = {}
_DESC_CACHE_MAX = 8192


def _arr(t: Optional[torch.Tensor]):
    """torch tensor -> pointer to a qw_array (None -> NULL)."""
    if t is None:
        return None
    key = (t.data_ptr(), t.dtype, t.shape, t.stride())
    d = _DESC_CACHE.get(key)
    if d is not None:
        return d
    if t.dtype not in _DT:
        raise TypeError(f"unsupported dtype {t.dtype}")
    if t.dim() < 1 or t.dim() > 4:
        raise ValueError("qw arrays have 1 to 4 dimensions")
    a = _lib.QwArray()
    a.data = t.data_ptr() if t.numel() else 0
    a.dtype = _DT[t.dtype]
    a.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        a.shape[i] = s
        a.strides[i] = st
    d = ctypes.pointer(a)
    if len(_DESC_CACHE) >= _DESC_CACHE_MAX:
        _DESC_CACHE.clear()
    _DESC_CACHE[key] = d
    return d


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _mode(mode: str) -> bytes:
    return mode.encode()


def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: Optional[torch.Tensor],
                     transpose: bool = True, group_size: int = 64, bits: int = 4, mode: str = "affine",
                     out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    """y = x @ dequantize(w, scales, biases).T  (lib.rs:1134-1143).

    ``out_dtype=torch.float32`` returns the fp32 accumulators unrounded (the
    partial sums of a row-parallel tensor-parallel shard)."""
    N = w.shape[0]
    if out is None:
        out = torch.empty(*x.shape[:-1], N, dtype=out_dtype, device=x.device)
    L = _lib.load()
    _lib.check(L.qw_quantized_matmul(_arr(x), _arr(w), _arr(scales), _arr(biases), int(bool(transpose)),
                                     group_size, bits, _mode(mode), _arr(out), _stream(x)))
    return out


def quantized_matmul_argmax(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: Optional[torch.Tensor],
                            group_size: int = 64, bits: int = 4, mode: str = "affine",
                            logits: Optional[torch.Tensor] = None,
                            idx: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Greedy token per row of x: argmax over the fp16 logits x @ dequantize(w).T
    (project_logits then argmax_last_axis, qwen3_5.rs:1038, lib.rs:2055).
    Returns uint32 indices as int64 (torch has no uint32 arithmetic); pass
    ``logits`` to also receive the fp16 logits (required above 16 rows).
    With ``idx`` (int32 [M], e.g. a buffer of a captured CUDA graph) the
    indices are written there as the ABI's uint32 and ``idx`` is returned."""
    M = x.numel() // x.shape[-1]
    out = idx if idx is not None else torch.empty(M, dtype=torch.int32, device=x.device)
    L = _lib.load()
    ia = _arr(out)  # int32 storage, passed as the uint32 ids the ABI returns
    _lib.check(L.qw_quantized_matmul_argmax(_arr(x), _arr(w), _arr(scales), _arr(biases), group_size, bits,
                                            _mode(mode), _arr(logits), ia, _stream(x)))
    if idx is not None:
        return idx
    return out.view(torch.int32).to(torch.int64) & 0xFFFFFFFF


def topk(logits: torch.Tensor, k: int, values: bool = True):
    """(indices int64 [..., k], values fp16 [..., k] or None): the k largest
    logits of each row, descending, lower index first among equal values --
    argpartition(logits, -k) + take_along_axis as top_k_candidate_logits
    (qwen3_5_dflash.rs:1236-1266) uses them, 1 <= k < N."""
    lead = logits.shape[:-1]
    idx = torch.empty(*lead, k, dtype=torch.int32, device=logits.device)
    val = torch.empty(*lead, k, dtype=torch.float16, device=logits.device) if values else None
    _lib.check(_lib.load().qw_topk(_arr(logits), int(k), _arr(idx), _arr(val), _stream(logits)))
    return idx.to(torch.int64) & 0xFFFFFFFF, val


def quantized_matmul_topk(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: Optional[torch.Tensor],
                          k: int, group_size: int = 64, bits: int = 4, mode: str = "affine",
                          logits: Optional[torch.Tensor] = None, values: bool = True):
    """The LM-head projection then the top k of each row (project_logits then
    top_k_candidate_logits, qwen3_5.rs:1038, qwen3_5_dflash.rs:1412);
    returns (indices int64, values fp16 or None).  ``logits`` (optional)
    receives the fp16 logits."""
    lead = x.shape[:-1]
    idx = torch.empty(*lead, k, dtype=torch.int32, device=x.device)
    val = torch.empty(*lead, k, dtype=torch.float16, device=x.device) if values else None
    _lib.check(_lib.load().qw_quantized_matmul_topk(_arr(x), _arr(w), _arr(scales), _arr(biases), group_size, bits,
                                                    _mode(mode), int(k), _arr(logits), _arr(idx), _arr(val),
                                                    _stream(x)))
    return idx.to(torch.int64) & 0xFFFFFFFF, val


def quantized_matmul_chain(ops, group_size: int = 64, bits: int = 4, mode: str = "affine") -> None:
    """Runs [(x, w, scales, biases, y), ...] in order, each y = x @ dequantize(w).T
    written into its preallocated ``y``; an op's x may be an earlier op's y.
    One cooperative launch per 24 ops when every x has at most 16 rows."""
    if not ops:
        return
    keep = []  # the descriptors must outlive the call
    arr = (_lib.QwQmmOp * len(ops))()
    for i, (x, w, s, b, y) in enumerate(ops):
        d = [_arr(x), _arr(w), _arr(s), _arr(b), _arr(y)]
        keep.append(d)
        arr[i].x, arr[i].w, arr[i].scales, arr[i].biases, arr[i].y = d
    L = _lib.load()
    _lib.check(L.qw_quantized_matmul_chain(arr, len(ops), group_size, bits, _mode(mode), _stream(ops[0][0])))


def quantized_matmul_swiglu(x: torch.Tensor, w_gate, scales_gate, biases_gate, w_up, scales_up, biases_up,
                            group_size: int = 64, bits: int = 4, mode: str = "affine",
                            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """silu(x @ dequantize(gate).T) * (x @ dequantize(up).T) in one kernel: the
    gate/up projections of Mlp::forward_hidden (qwen3_next.rs:463-487) and
    compiled_swiglu_activation (mlx_cxx_bridge.cpp:1205-1216), with the
    reference's fp16 rounding after each op."""
    if out is None:
        out = torch.empty(*x.shape[:-1], w_gate.shape[0], dtype=torch.float16, device=x.device)
    L = _lib.load()
    _lib.check(L.qw_quantized_matmul_swiglu(_arr(x), _arr(w_gate), _arr(scales_gate), _arr(biases_gate),
                                            _arr(w_up), _arr(scales_up), _arr(biases_up), 1, group_size, bits,
                                            _mode(mode), _arr(out), _stream(x)))
    return out


def compiled_swiglu_activation(gate: torch.Tensor, up: torch.Tensor, out: Optional[torch.Tensor] = None):
    """silu(gate) * up on fp16 tensors (lib.rs:627, mlx_cxx_bridge.cpp:1255)."""
    if out is None:
        out = torch.empty_like(gate)
    _lib.check(_lib.load().qw_swiglu_activation(_arr(gate), _arr(up), _arr(out), _stream(gate)))
    return out


def swiglu_mlp(x: torch.Tensor, w_gate, scales_gate, biases_gate, w_up, scales_up, biases_up, w_down, scales_down,
               biases_down, group_size: int = 64, bits: int = 4, mode: str = "affine",
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """down(silu(gate(x)) * up(x)) for quantized projections: the reference's
    compiled_moe_expert_forward (lib.rs:1636-1652, mlx_cxx_bridge.cpp:4238)."""
    if out is None:
        out = torch.empty(*x.shape[:-1], w_down.shape[0], dtype=torch.float16, device=x.device)
    L = _lib.load()
    _lib.check(L.qw_swiglu_mlp(_arr(x), _arr(w_gate), _arr(scales_gate), _arr(biases_gate), _arr(w_up),
                               _arr(scales_up), _arr(biases_up), _arr(w_down), _arr(scales_down),
                               _arr(biases_down), group_size, bits, _mode(mode), _arr(out), _stream(x)))
    return out


compiled_moe_expert_forward = swiglu_mlp


def quantized_linear_forward(x, w, scales, biases, linear_bias=None, group_size: int = 64, bits: int = 4,
                             mode: str = "affine", out=None) -> torch.Tensor:
    """Quantized linear layer forward (lib.rs:591-601)."""
    if out is None:
        out = torch.empty(*x.shape[:-1], w.shape[0], dtype=torch.float16, device=x.device)
    L = _lib.load()
    _lib.check(L.qw_quantized_linear_forward(_arr(x), _arr(w), _arr(scales), _arr(biases), _arr(linear_bias),
                                             group_size, bits, _mode(mode), _arr(out), _stream(x)))
    return out


def quantized_linear_forward_global_scale(x, w, scales, biases, global_scale=None, linear_bias=None,
                                          group_size: int = 64, bits: int = 4, mode: str = "affine",
                                          out=None) -> torch.Tensor:
    """Quantized linear forward with a post-qmm global scale (lib.rs:604-615)."""
    if out is None:
        out = torch.empty(*x.shape[:-1], w.shape[0], dtype=torch.float16, device=x.device)
    L = _lib.load()
    _lib.check(L.qw_quantized_linear_forward_global_scale(
        _arr(x), _arr(w), _arr(scales), _arr(biases), _arr(global_scale), _arr(linear_bias), group_size, bits,
        _mode(mode), _arr(out), _stream(x)))
    return out


def dequantize(w, scales, biases, group_size: int = 64, bits: int = 4, mode: str = "affine",
               rounding: int = 0, out=None) -> torch.Tensor:
    """Full-precision weights from the quantized triple (lib.rs:1152-1159).

    rounding 0: fp16(fp16(s*q) + b); rounding 1: fp16(s*q + b) rounded once."""
    K = w.shape[1] * 32 // bits
    if out is None:
        out = torch.empty(w.shape[0], K, dtype=torch.float16, device=w.device)
    L = _lib.load()
    _lib.check(L.qw_dequantize_rounding(_arr(w), _arr(scales), _arr(biases), group_size, bits, _mode(mode),
                                        rounding, _arr(out), _stream(w)))
    return out


def quantize_weights(w: torch.Tensor, group_size: int = 64, bits: int = 4,
                     mode: str = "affine") -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Quantize once and return the (w, scales, biases) triple (lib.rs:2707-2742)."""
    N, K = w.shape
    wq = torch.empty(N, K * bits // 32, dtype=torch.int32, device=w.device)
    s = torch.empty(N, K // group_size, dtype=torch.float16, device=w.device)
    b = torch.empty(N, K // group_size, dtype=torch.float16, device=w.device)
    L = _lib.load()
    _lib.check(L.qw_quantize(_arr(w), group_size, bits, _mode(mode), _arr(wq), _arr(s), _arr(b), _stream(w)))
    return wq, s, b


def decode_schedule(M: int, N: int, K: int, bits: int = 4, group_size: int = 64, swiglu: bool = False,
                    sm_count: int = 148) -> dict:
    """The decode kernel's configuration and schedule for a matmul of M (1..16)
    rows of x against an N x K weight (qw_decode_schedule; no device access)."""
    out = (ctypes.c_int64 * 5)()
    _lib.check(_lib.load().qw_decode_schedule(int(M), int(N), int(K), bits, group_size, int(bool(swiglu)),
                                              int(sm_count), out))
    return {"tokens": out[0], "unit_k": out[1], "ctas": out[2], "split": out[3], "busiest_units": out[4]}


def device_status(device: int = 0, clear: bool = True) -> int:
    """Device-side status word left by a kernel whose bounded wait ran out (0 = none)."""
    v = ctypes.c_uint(0)
    rc = _lib.load().qw_device_status(device, ctypes.byref(v), int(clear))
    if rc not in (_lib.QW_OK, _lib.QW_ETIMEOUT):
        _lib.check(rc)
    return int(v.value)


class QuantizedLinear:
    """A quantized weight triple and its forward, after mlxcel-core's
    ``QuantizedWeight`` (layers.rs:35-174) and the quantized arm of
    ``UnifiedLinear::forward`` (layers.rs:2023-2093)."""

    def __init__(self, w, scales, biases, group_size: int = 64, bits: int = 4, mode: str = "affine",
                 bias: Optional[torch.Tensor] = None, global_scale: Optional[torch.Tensor] = None):
        self.weight, self.scales, self.biases = w, scales, biases
        self.group_size, self.bits, self.mode = group_size, bits, mode
        self.bias = bias
        self.global_scale = global_scale

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    @property
    def in_features(self) -> int:
        return self.weight.shape[1] * 32 // self.bits

    def forward(self, x: torch.Tensor, out=None) -> torch.Tensor:
        if self.global_scale is not None:
            return quantized_linear_forward_global_scale(x, self.weight, self.scales, self.biases,
                                                         self.global_scale, self.bias, self.group_size,
                                                         self.bits, self.mode, out=out)
        return quantized_linear_forward(x, self.weight, self.scales, self.biases, self.bias, self.group_size,
                                        self.bits, self.mode, out=out)

    __call__ = forward


class QuantizedFusedLinear:
    """Projections of one input fused into one quantized matmul: the planes'
    weights, scales and biases concatenated along the output rows, the output
    split back into column views (no copies).  After the reference's
    FusedQKVLinear (layers.rs:2467-2850: q|k|v concatenated at load,
    ``forward`` returning (q, k, v)), the GDN z|b|a input projections
    (qwen3_5.rs:383-435) and the gate|up fusion (qwen3_next.rs:406-447).
    The views are row-strided when there are several rows; the library's
    matmuls accept them as x directly."""

    def __init__(self, linear: QuantizedLinear, sizes):
        if sum(sizes) != linear.out_features:
            raise ValueError(f"plane sizes {list(sizes)} do not add up to {linear.out_features} rows")
        self.linear, self.sizes = linear, tuple(int(n) for n in sizes)

    @classmethod
    def from_linears(cls, linears):
        """Concatenate quantized linears that share input width, group size,
        bits and mode (and have no linear bias or global scale)."""
        first = linears[0]
        for l in linears:
            if (l.in_features, l.group_size, l.bits, l.mode) != (first.in_features, first.group_size, first.bits,
                                                                 first.mode):
                raise ValueError("fused planes must share input width and quantization")
            if l.bias is not None or l.global_scale is not None:
                raise ValueError("fused planes take no linear bias or global scale")
        cat = lambda ts: torch.cat(ts, 0).contiguous()  # noqa: E731
        fused = QuantizedLinear(cat([l.weight for l in linears]), cat([l.scales for l in linears]),
                                cat([l.biases for l in linears]) if first.biases is not None else None,
                                first.group_size, first.bits, first.mode)
        return cls(fused, [l.out_features for l in linears])

    def forward(self, x: torch.Tensor, out=None):
        y = self.linear(x, out=out)
        views, c = [], 0
        for n in self.sizes:
            views.append(y[..., c:c + n])
            c += n
        return tuple(views)

    __call__ = forward


class QuantizedMlp:
    """Dense SwiGLU MLP over three QuantizedLinear projections, after the
    reference's ``Mlp`` (qwen3_next.rs:449-487).  The gate and up projections
    run as one fused kernel when ``fuse_mlp_input_projections``
    (qwen3_next.rs:406-447) would fuse them: same group size, bits and mode,
    no linear biases and no global scales; otherwise as two matmuls followed
    by the activation (the reference's Separate arm).  A checkpoint that
    stores them concatenated is split into two row views by ``from_fused``."""

    def __init__(self, gate: QuantizedLinear, up: QuantizedLinear, down: QuantizedLinear):
        self.gate, self.up, self.down = gate, up, down
        self.fused = (gate.group_size == up.group_size and gate.bits == up.bits and gate.mode == up.mode
                      and gate.bias is None and up.bias is None
                      and gate.global_scale is None and up.global_scale is None
                      and gate.out_features == up.out_features)

    @classmethod
    def from_fused(cls, gate_up: QuantizedLinear, intermediate_size: int, down: QuantizedLinear):
        """Gate and up stored as one [2I, ...] projection (rows 0..I-1 gate)."""
        def half(t, i):
            return None if t is None else t[i * intermediate_size:(i + 1) * intermediate_size]
        g = QuantizedLinear(half(gate_up.weight, 0), half(gate_up.scales, 0), half(gate_up.biases, 0),
                            gate_up.group_size, gate_up.bits, gate_up.mode)
        u = QuantizedLinear(half(gate_up.weight, 1), half(gate_up.scales, 1), half(gate_up.biases, 1),
                            gate_up.group_size, gate_up.bits, gate_up.mode)
        return cls(g, u, down)

    def forward_hidden(self, x: torch.Tensor, out=None) -> torch.Tensor:
        g, u = self.gate, self.up
        if self.fused:
            return quantized_matmul_swiglu(x, g.weight, g.scales, g.biases, u.weight, u.scales, u.biases,
                                           g.group_size, g.bits, g.mode, out=out)
        return compiled_swiglu_activation(g(x), u(x), out=out)

    def forward(self, x: torch.Tensor, out=None) -> torch.Tensor:
        return self.down(self.forward_hidden(x), out=out)

    __call__ = forward
