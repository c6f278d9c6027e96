"""A checkpoint written in MLX's safetensors format, loaded by qw_b200.loader
and run through the library's kernels, against the CPU oracle on the same
bytes.  Tolerance: max |y - y_ref| <= 1e-2 * rms(y_ref)."""
import json

import numpy as np
import pytest
import torch

import oracle
from qw_b200 import _lib, loader, synth
from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


def test_loaded_linears_match_the_oracle(tmp_path, cuda_dev):
    shapes = {"model.layers.0.mlp.gate_up_proj": (1024, 512), "model.layers.0.mlp.down_proj": (512, 2048),
              "lm_head": (1000, 512)}
    arrays = {}
    for i, (prefix, (N, K)) in enumerate(shapes.items()):
        wq, s, b = oracle.quantize(synth.weight_fp16(N, K, seed=40 + i))
        arrays.update({prefix + ".weight": wq, prefix + ".scales": s, prefix + ".biases": b})
    loader.write_safetensors(str(tmp_path / "model.safetensors"), arrays)
    (tmp_path / "config.json").write_text(json.dumps({"quantization": {"group_size": 64, "bits": 4,
                                                                        "mode": "affine"}}))
    ck = loader.Checkpoint(str(tmp_path))
    for prefix, (N, K) in shapes.items():
        lin = ck.quantized(prefix).to_device()
        for M in (1, 7, 40):
            x = synth.activations(M, K, seed=M)
            y = lin(torch.from_numpy(x).cuda())
            torch.cuda.synchronize()
            _, y_ref = oracle.quantized_matmul(x, arrays[prefix + ".weight"], arrays[prefix + ".scales"],
                                               arrays[prefix + ".biases"], want_f32=True)
            assert rel_err(y.float().cpu().numpy(), y_ref) <= TOL, (prefix, M)


def test_overrides_run_or_fail_loudly(tmp_path, cuda_dev):
    """An 8-bit override runs through the kernels; a 2-bit one (which MLX
    accepts and this library does not implement) raises QW_EUNSUPPORTED."""
    w8 = oracle.quantize(synth.weight_fp16(64, 512, seed=1), group_size=64, bits=8)
    w2 = oracle.quantize(synth.weight_fp16(64, 512, seed=2), group_size=64, bits=2)
    loader.write_safetensors(str(tmp_path / "model.safetensors"), {
        "g8.weight": w8[0], "g8.scales": w8[1], "g8.biases": w8[2],
        "g2.weight": w2[0], "g2.scales": w2[1], "g2.biases": w2[2]})
    (tmp_path / "config.json").write_text(json.dumps({"quantization": {
        "group_size": 64, "bits": 4, "mode": "affine",
        "g8": {"group_size": 64, "bits": 8}, "g2": {"group_size": 64, "bits": 2}}}))
    ck = loader.Checkpoint(str(tmp_path))
    x = synth.activations(3, 512, seed=3)
    y = ck.quantized("g8").to_device()(torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    _, y_ref = oracle.quantized_matmul(x, *w8, group_size=64, bits=8, want_f32=True)
    assert rel_err(y.float().cpu().numpy(), y_ref) <= TOL
    lin = ck.quantized("g2").to_device()
    with pytest.raises(_lib.QwError) as e:
        lin(torch.zeros(1, 512, dtype=torch.float16, device="cuda"))
    assert e.value.code == _lib.QW_EUNSUPPORTED
