"""Top-k candidates (qw_topk, qw_quantized_matmul_topk) against the oracle's
restatement: exact index and value equality, since selection on fp16 logits
involves no arithmetic.  Cases: the reference's candidate vectors (four peaks
over a flat floor), random rows at the vocabulary sizes of the model (248,320)
and of BASELINE's stack (151,936), heavy ties at the k-th value (coarse
values, all-equal rows), signed zeros, k from 1 to 1024 and N - 1, and the
bounds the reference's caller checks."""
import numpy as np
import pytest
import torch

import oracle
import qw_b200
from qw_b200 import _lib, synth
from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check(logits, k):
    idx, vals = qw_b200.topk(dev(logits), k)
    torch.cuda.synchronize()
    ridx, rvals = oracle.topk(logits, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_array_equal(vals.cpu().numpy().view(np.uint16), rvals.view(np.uint16))


def test_reference_candidate_vectors(cuda_dev):
    peaks = {0: 40.0, 80_000: 50.0, 80_001: 60.0, 80_921: 70.0}
    for n, floor in ((80_922, -1000.0), (248_320, -2000.0)):
        logits = np.full((1, 1, n), floor, np.float16)
        for i, v in peaks.items():
            logits[0, 0, i] = v
        check(logits, 4)


@pytest.mark.parametrize("N", [248_320, 151_936, 5000])
@pytest.mark.parametrize("k", [1, 16, 64, 1024])
def test_random_rows(cuda_dev, N, k):
    rng = np.random.default_rng(N + k)
    logits = (rng.standard_normal((16, N)) * 3).astype(np.float16)
    check(logits, k)


@pytest.mark.parametrize("k", [1, 7, 16, 300, 1024])
def test_ties_at_the_boundary(cuda_dev, k):
    """Coarse values: many logits share the k-th value, so the lowest indices
    among them must be the ones taken."""
    rng = np.random.default_rng(k)
    logits = rng.integers(-4, 5, size=(5, 248_320)).astype(np.float16)
    logits[1] = 2.0  # a row of equal values
    logits[2, ::2] = -0.0
    logits[2, 1::2] = 0.0
    check(logits, k)


def test_small_rows_and_k_near_n(cuda_dev):
    rng = np.random.default_rng(3)
    for n in (2, 3, 17, 1024, 1025, 4097):
        logits = rng.standard_normal((3, n)).astype(np.float16)
        for k in sorted({1, min(n // 2 or 1, 1024), min(n - 1, 1024)}):
            check(logits, k)


def test_bounds(cuda_dev):
    z = dev(np.zeros((1, 1, 4), np.float16))
    for bad in (0, 4, 5):
        with pytest.raises(_lib.QwError, match="must be in 1..3"):
            qw_b200.topk(z, bad)
    big = dev(np.zeros((1, 5000), np.float16))
    with pytest.raises(_lib.QwError, match="supported"):
        qw_b200.topk(big, 1025)


@pytest.mark.parametrize("M", [1, 16, 40])
def test_projection_topk(cuda_dev, M):
    """LM-head projection then top-k (the DFlash2 candidate step): the indices
    and values are exactly the top-k of the logits the call wrote, and the
    logits are within tolerance of the oracle's; also without a logits buffer."""
    N, K, k = 6000, 1024, 16
    wq, s, b = oracle.quantize(synth.weight_fp16(N, K, seed=M))
    x = synth.activations(M, K, seed=M + 1)
    W, S, B = (torch.from_numpy(np.ascontiguousarray(wq).view(np.int32)).cuda(), dev(s), dev(b))
    logits = torch.empty(M, N, dtype=torch.float16, device="cuda")
    idx, vals = qw_b200.quantized_matmul_topk(dev(x), W, S, B, k, logits=logits)
    idx2, vals2 = qw_b200.quantized_matmul_topk(dev(x), W, S, B, k)
    torch.cuda.synchronize()
    lg = logits.cpu().numpy()
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    assert rel_err(lg, y_ref) <= TOL
    ridx, rvals = oracle.topk(lg, k)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_array_equal(vals.cpu().numpy().view(np.uint16), rvals.view(np.uint16))
    np.testing.assert_array_equal(idx2.cpu().numpy(), ridx)
    np.testing.assert_array_equal(vals2.cpu().numpy().view(np.uint16), rvals.view(np.uint16))
