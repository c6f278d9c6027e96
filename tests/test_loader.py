"""MLX-format quantized checkpoints (qw_b200.loader) on CPU: headers, shards,
per-tensor quantization overrides and the load-time checks QW applies.  The
GPU forward of a loaded linear is in test_gpu_loader.py."""
import json
import os
import struct

import numpy as np
import pytest

import oracle
from qw_b200 import loader, synth


def _quant(N, K, seed, gs=64, bits=4):
    w = synth.weight_fp16(N, K, seed=seed)
    if (gs, bits) == (64, 4):
        return oracle.quantize(w)
    return oracle.quantize(w, group_size=gs, bits=bits)


def _write_checkpoint(tmp_path, sharded=True, config=True):
    lins = {
        "model.layers.0.self_attn.q_proj": (384, 512, 64, 4),
        "model.layers.0.mlp.down_proj": (256, 1024, 64, 4),
        "model.layers.1.mlp.gate": (64, 512, 64, 8),      # override: 8-bit
        "model.layers.1.mlp.up_proj": (128, 512, 128, 4),  # override via the language_model. name
    }
    arrays = {}
    for i, (prefix, (N, K, gs, bits)) in enumerate(lins.items()):
        wq, s, b = _quant(N, K, seed=i, gs=gs, bits=bits)
        arrays[prefix + ".weight"] = wq
        arrays[prefix + ".scales"] = s
        arrays[prefix + ".biases"] = b
    arrays["model.norm.weight"] = np.ones(512, np.float16)
    names = list(arrays)
    if sharded:
        half = len(names) // 2
        shards = {"model-00001-of-00002.safetensors": names[:half],
                  "model-00002-of-00002.safetensors": names[half:]}
        for fname, ns in shards.items():
            loader.write_safetensors(str(tmp_path / fname), {n: arrays[n] for n in ns}, metadata={"format": "mlx"})
        index = {"metadata": {"total_size": 0}, "weight_map": {n: f for f, ns in shards.items() for n in ns}}
        (tmp_path / "model.safetensors.index.json").write_text(json.dumps(index))
    else:
        loader.write_safetensors(str(tmp_path / "model.safetensors"), arrays)
    if config:
        cfg = {"model_type": "qwen3_5", "quantization": {
            "group_size": 64, "bits": 4, "mode": "affine",
            "model.layers.1.mlp.gate": {"group_size": 64, "bits": 8},
            "language_model.model.layers.1.mlp.up_proj": {"group_size": 128, "bits": 4}}}
        (tmp_path / "config.json").write_text(json.dumps(cfg))
    return arrays, lins


@pytest.mark.parametrize("sharded", [True, False])
def test_tensors_round_trip(tmp_path, sharded):
    arrays, _ = _write_checkpoint(tmp_path, sharded=sharded)
    ck = loader.Checkpoint(str(tmp_path))
    assert set(ck.names()) == set(arrays)
    for name, a in arrays.items():
        got = ck.array(name)
        assert got.dtype == a.dtype and got.shape == a.shape
        np.testing.assert_array_equal(got, a)


def test_quantization_overrides_follow_quant_params(tmp_path):
    _write_checkpoint(tmp_path)
    q = loader.Checkpoint(str(tmp_path)).quant
    assert q.params("model.layers.0.self_attn.q_proj") == (64, 4)      # the default
    assert q.params("model.layers.1.mlp.gate") == (64, 8)              # override by prefix
    assert q.params("model.layers.1.mlp.up_proj") == (128, 4)          # override by language_model.prefix
    assert loader.QuantConfig(None).params("anything") == (64, 4)      # no quantization object


def test_quantized_linear_tensors_and_matmul(tmp_path):
    arrays, lins = _write_checkpoint(tmp_path)
    ck = loader.Checkpoint(str(tmp_path))
    for prefix, (N, K, gs, bits) in lins.items():
        qt = ck.quantized(prefix)
        assert (qt.group_size, qt.bits) == (gs, bits)
        assert qt.out_features == N and qt.in_features == K
    qt = ck.quantized("model.layers.0.self_attn.q_proj")
    x = synth.activations(2, 512, seed=1)
    y_loaded = oracle.quantized_matmul(x, qt.weight, qt.scales, qt.biases)
    pfx = "model.layers.0.self_attn.q_proj"
    y_orig = oracle.quantized_matmul(x, arrays[pfx + ".weight"], arrays[pfx + ".scales"], arrays[pfx + ".biases"])
    np.testing.assert_array_equal(y_loaded.view(np.uint16), y_orig.view(np.uint16))


def test_packing_invariant_and_missing_biases_are_rejected(tmp_path):
    wq, s, b = _quant(128, 512, seed=3)
    loader.write_safetensors(str(tmp_path / "model.safetensors"), {
        "a.weight": wq, "a.scales": s, "a.biases": b,
        "bad.weight": wq[:, :60], "bad.scales": s, "bad.biases": b,      # packed width != groups
        "nob.weight": wq, "nob.scales": s,                                 # affine without biases
        "f32.weight": wq.view(np.float32), "f32.scales": s, "f32.biases": b,
    })
    ck = loader.Checkpoint(str(tmp_path))
    ck.quantized("a")
    with pytest.raises(loader.CheckpointError, match="packed width"):
        ck.quantized("bad")
    with pytest.raises(loader.CheckpointError, match="requires biases"):
        ck.quantized("nob")
    with pytest.raises(loader.CheckpointError, match="U32"):
        ck.quantized("f32")
    with pytest.raises(loader.CheckpointError, match="missing tensor"):
        ck.quantized("absent")


def test_corrupt_headers_are_rejected(tmp_path):
    p = tmp_path / "model.safetensors"
    p.write_bytes(struct.pack("<Q", 0))
    with pytest.raises(loader.CheckpointError, match="implausible"):
        loader.read_header(str(p))
    p.write_bytes(struct.pack("<Q", 10) + b"not json!!")
    with pytest.raises(loader.CheckpointError, match="not JSON"):
        loader.read_header(str(p))
    hdr = json.dumps({"t": {"dtype": "F16", "shape": [4], "data_offsets": [0, 6]}}).encode()
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 8)
    with pytest.raises(loader.CheckpointError, match="data_offsets"):
        loader.read_header(str(p))
    hdr = json.dumps({"t": {"dtype": "C64", "shape": [1], "data_offsets": [0, 8]}}).encode()
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + b"\0" * 8)
    with pytest.raises(loader.CheckpointError, match="unsupported dtype"):
        loader.read_header(str(p))


def test_stale_index_falls_back_to_the_files_on_disk(tmp_path):
    arrays, _ = _write_checkpoint(tmp_path, sharded=False)
    (tmp_path / "model.safetensors.index.json").write_text(
        json.dumps({"weight_map": {"x": "model-00001-of-00009.safetensors"}}))
    ck = loader.Checkpoint(str(tmp_path))
    assert set(ck.names()) == set(arrays)


def test_empty_directory_is_an_error(tmp_path):
    with pytest.raises(loader.CheckpointError, match="no safetensors"):
        loader.Checkpoint(str(tmp_path))
