"""MLX-format quantized checkpoints (safetensors) for the quantized linears.

What QW's loader reads for a quantized linear `prefix` (crates/mlxcel-core/src/
weights.rs, crates/runtime/src/qwen3_next.rs):

* `prefix.weight`  U32 [N, K*bits/32], codes packed along K (weights.rs:150-158);
* `prefix.scales`  F16 [N, K/group_size];
* `prefix.biases`  F16 [N, K/group_size] (affine mode);
* the checkpoint's `config.json` "quantization" object: `group_size`, `bits`,
  `mode`, and per-tensor overrides keyed by the linear's prefix, looked up
  as the prefix and then as "language_model." + prefix
  (Qwen3NextConfig::quant_params, qwen3_next.rs:60-72; (64, 4) when the
  config has no quantization object).

The files are found as weights.rs does: the shard list of
`model.safetensors.index.json` when it exists and every shard it names is on
disk, otherwise every `*.safetensors` file in the directory
(weights.rs:380-420).  A safetensors file is an 8-byte little-endian header
length, a JSON header mapping tensor names to {dtype, shape, data_offsets}
(offsets relative to the end of the header; the "__metadata__" entry is not a
tensor), then the tensor bytes.

Tensors are memory-mapped and copied to the device only when asked for.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np

_DTYPES = {
    "F64": np.float64, "F32": np.float32, "F16": np.float16, "I64": np.int64, "I32": np.int32,
    "U32": np.uint32, "I16": np.int16, "U16": np.uint16, "I8": np.int8, "U8": np.uint8, "BOOL": np.bool_,
}
MAX_HEADER_BYTES = 256 * 1024 * 1024


class CheckpointError(ValueError):
    """A checkpoint that does not describe valid quantized linears."""


@dataclass(frozen=True)
class TensorEntry:
    path: str
    dtype: str
    shape: Tuple[int, ...]
    begin: int  # absolute byte offset in the file
    end: int


def read_header(path: str) -> Dict[str, TensorEntry]:
    """Tensor table of one safetensors file (no tensor data is read)."""
    with open(path, "rb") as f:
        raw = f.read(8)
        if len(raw) != 8:
            raise CheckpointError(f"{path}: shorter than a safetensors header")
        (n,) = struct.unpack("<Q", raw)
        if n == 0 or n > MAX_HEADER_BYTES:
            raise CheckpointError(f"{path}: implausible header length {n}")
        header = f.read(n)
        if len(header) != n:
            raise CheckpointError(f"{path}: truncated header")
        size = os.fstat(f.fileno()).st_size
    try:
        table = json.loads(header.decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError) as e:
        raise CheckpointError(f"{path}: header is not JSON ({e})") from None
    if not isinstance(table, dict):
        raise CheckpointError(f"{path}: header is not a JSON object")
    out: Dict[str, TensorEntry] = {}
    base = 8 + n
    for name, meta in table.items():
        if name == "__metadata__":
            continue
        try:
            dtype, shape, (b, e) = meta["dtype"], tuple(int(d) for d in meta["shape"]), meta["data_offsets"]
        except (KeyError, TypeError, ValueError):
            raise CheckpointError(f"{path}: malformed entry for {name!r}") from None
        if dtype not in _DTYPES:
            raise CheckpointError(f"{path}: {name!r} has unsupported dtype {dtype}")
        nbytes = int(np.prod(shape, dtype=np.int64)) * np.dtype(_DTYPES[dtype]).itemsize
        if e - b != nbytes or b < 0 or base + e > size:
            raise CheckpointError(f"{path}: {name!r} data_offsets {b}..{e} do not match {dtype}{list(shape)}")
        out[name] = TensorEntry(path, dtype, shape, base + int(b), base + int(e))
    return out


def shard_paths(directory: str) -> List[str]:
    """The checkpoint's safetensors files: the index's shards if all exist, else a glob."""
    index = os.path.join(directory, "model.safetensors.index.json")
    globbed = sorted(os.path.join(directory, f) for f in os.listdir(directory) if f.endswith(".safetensors"))
    if os.path.exists(index):
        with open(index) as f:
            names = sorted(set(json.load(f).get("weight_map", {}).values()))
        paths = [os.path.join(directory, n) for n in names]
        if names and all(os.path.exists(p) for p in paths):
            return paths
        if globbed:
            return globbed  # a repackaged checkpoint whose index names other shards
        missing = [p for p in paths if not os.path.exists(p)]
        raise CheckpointError(f"{directory}: index names missing shards {missing[:3]}")
    if not globbed:
        raise CheckpointError(f"{directory}: no safetensors files")
    return globbed


class QuantConfig:
    """config.json's "quantization" object with per-tensor overrides."""

    def __init__(self, quantization: Optional[dict]):
        self.q = quantization

    def params(self, prefix: str) -> Tuple[int, int]:
        """(group_size, bits) for the linear `prefix` (qwen3_next.rs:60-72)."""
        if self.q is None:
            return 64, 4
        for key in (prefix, "language_model." + prefix):
            o = self.q.get(key)
            if isinstance(o, dict) and "group_size" in o and "bits" in o:
                return int(o["group_size"]), int(o["bits"])
        return int(self.q["group_size"]), int(self.q["bits"])

    @property
    def mode(self) -> str:
        return (self.q or {}).get("mode", "affine")


class Checkpoint:
    """A directory of MLX-format safetensors shards and its config.json."""

    def __init__(self, directory: str):
        self.directory = directory
        self.tensors: Dict[str, TensorEntry] = {}
        for path in shard_paths(directory):
            for name, entry in read_header(path).items():
                if name in self.tensors:
                    raise CheckpointError(f"{name!r} appears in two shards")
                self.tensors[name] = entry
        cfg_path = os.path.join(directory, "config.json")
        cfg = {}
        if os.path.exists(cfg_path):
            with open(cfg_path) as f:
                cfg = json.load(f)
        self.config = cfg
        self.quant = QuantConfig(cfg.get("quantization") or cfg.get("quantization_config"))
        self._maps: Dict[str, np.memmap] = {}

    def names(self) -> Iterable[str]:
        return self.tensors.keys()

    def array(self, name: str) -> np.ndarray:
        """The tensor as a read-only numpy view of the memory-mapped file."""
        e = self.tensors.get(name)
        if e is None:
            raise CheckpointError(f"missing tensor {name!r}")
        mm = self._maps.get(e.path)
        if mm is None:
            mm = self._maps[e.path] = np.memmap(e.path, dtype=np.uint8, mode="r")
        return mm[e.begin:e.end].view(_DTYPES[e.dtype]).reshape(e.shape)

    def quantized(self, prefix: str) -> "QuantizedTensors":
        """The packed weight, scales and biases of linear `prefix`, checked."""
        group_size, bits = self.quant.params(prefix)
        w = self.array(prefix + ".weight")
        s = self.array(prefix + ".scales")
        mode = self.quant.mode
        b = self.array(prefix + ".biases") if prefix + ".biases" in self.tensors else None
        if self.tensors[prefix + ".weight"].dtype != "U32":
            raise CheckpointError(f"{prefix}.weight must be U32, got {self.tensors[prefix + '.weight'].dtype}")
        if w.ndim != 2 or s.ndim != 2 or s.shape[0] != w.shape[0]:
            raise CheckpointError(f"{prefix}: weight {w.shape} and scales {s.shape} disagree on rows")
        # packing invariant (layers.rs:1568-1570): packed_in * 32 == bits * groups * group_size
        if w.shape[1] * 32 != bits * s.shape[1] * group_size:
            raise CheckpointError(f"{prefix}: packed width {w.shape[1]} at {bits}-bit does not match "
                                  f"{s.shape[1]} groups of {group_size}")
        if mode == "affine" and b is None:
            raise CheckpointError(f"{prefix}: affine quantization requires biases")
        if b is not None and b.shape != s.shape:
            raise CheckpointError(f"{prefix}: biases {b.shape} must match scales {s.shape}")
        return QuantizedTensors(prefix, w, s, b, group_size, bits, mode)


@dataclass
class QuantizedTensors:
    prefix: str
    weight: np.ndarray   # uint32 [N, K*bits/32]
    scales: np.ndarray   # float16 [N, G]
    biases: Optional[np.ndarray]
    group_size: int
    bits: int
    mode: str

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    @property
    def in_features(self) -> int:
        return self.weight.shape[1] * 32 // self.bits

    def to_device(self, device="cuda"):
        """A QuantizedLinear on `device` (the library's kernels; unsupported
        (bits, group_size) pairs raise from the C ABI on first use)."""
        import torch
        from .ops import QuantizedLinear

        def dev(a, dt):
            # the memory-mapped views are read-only: stage a writable host copy
            return torch.from_numpy(np.require(a, requirements=["C", "W"]).view(dt)).to(device)

        wq = dev(self.weight, np.int32)
        s = dev(self.scales, np.float16)
        b = dev(self.biases, np.float16) if self.biases is not None else None
        return QuantizedLinear(wq, s, b, group_size=self.group_size, bits=self.bits, mode=self.mode)


def write_safetensors(path: str, tensors: Dict[str, np.ndarray], metadata: Optional[Dict[str, str]] = None):
    """Write a safetensors file (for tests and for exporting checkpoints)."""
    rev = {np.dtype(v): k for k, v in _DTYPES.items()}
    header: Dict[str, object] = {}
    if metadata:
        header["__metadata__"] = dict(metadata)
    offset = 0
    blobs = []
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        nb = a.nbytes
        header[name] = {"dtype": rev[a.dtype], "shape": list(a.shape), "data_offsets": [offset, offset + nb]}
        blobs.append(a.tobytes())
        offset += nb
    raw = json.dumps(header).encode("utf-8")
    raw += b" " * ((8 - len(raw) % 8) % 8)  # keep the data 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for blob in blobs:
            f.write(blob)
