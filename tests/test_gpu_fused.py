"""Fused projections (QuantizedFusedLinear): q|k|v concatenated at load and
run as one matmul whose output splits into column views, as the reference's
FusedQKVLinear does (layers.rs:2467-2850); each view matches the oracle of
its own plane, and a view feeds the next matmul as a row-strided x."""
import numpy as np
import pytest
import torch

import oracle
import qw_b200
from qw_b200 import synth
from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def lin(p, bits=4, gs=64):
    wq, s, b = p
    return qw_b200.QuantizedLinear(dev(np.ascontiguousarray(wq).view(np.int32)), dev(s), dev(b),
                                   group_size=gs, bits=bits)


@pytest.mark.parametrize("M", [1, 5, 40])
def test_qkv_views_match_planes(cuda_dev, M):
    K = 512
    planes = [oracle.quantize(synth.weight_fp16(n, K, seed=i)) for i, n in enumerate((384, 64, 64))]
    fused = qw_b200.QuantizedFusedLinear.from_linears([lin(p) for p in planes])
    x = synth.activations(M, K, seed=M)
    q, k, v = fused(dev(x))
    # o-like projection consuming the q view without a copy (row-strided when M > 1)
    o = oracle.quantize(synth.weight_fp16(128, 384, seed=9))
    y = lin(o)(q)
    torch.cuda.synchronize()
    for view, p in zip((q, k, v), planes):
        _, ref = oracle.quantized_matmul(x, *p, want_f32=True)
        assert view.shape == (M, p[0].shape[0])
        assert rel_err(view.cpu().numpy(), ref) <= TOL
    _, y_ref = oracle.quantized_matmul(q.cpu().numpy(), *o, want_f32=True)
    assert rel_err(y.cpu().numpy(), y_ref) <= TOL


def test_mismatched_planes_are_rejected(cuda_dev):
    a = lin(oracle.quantize(synth.weight_fp16(64, 512, seed=1)))
    b8 = lin(oracle.quantize(synth.weight_fp16(64, 512, seed=2), bits=8), bits=8)
    with pytest.raises(ValueError, match="share"):
        qw_b200.QuantizedFusedLinear.from_linears([a, b8])
    with pytest.raises(ValueError, match="add up"):
        qw_b200.QuantizedFusedLinear(a, [32, 16])
