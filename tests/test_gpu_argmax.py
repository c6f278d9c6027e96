"""qw_quantized_matmul_argmax: the greedy token of a projection.

The fused path (M <= 16: keys folded into the skinny kernel's epilogue) must
return exactly the first index of the maximum of the fp16 logits that
qw_quantized_matmul produces for the same inputs; the M > 16 path runs the
prefill matmul and a row argmax.  Ties resolve to the lowest index, and the
chosen logit is the oracle's maximum within the output tolerance."""
import numpy as np
import pytest
import torch

import oracle
import qw_b200
from qw_b200 import _lib, synth
from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


def _weights(N, K, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return qw_b200.quantize_weights((torch.randn(N, K, generator=g, device="cuda") * 0.02).half())


@pytest.mark.parametrize("M", [1, 4, 16])
@pytest.mark.parametrize("N,K", [(151936, 5120), (1000, 512), (130, 576)])
def test_argmax_matches_logits(cuda_dev, M, N, K):
    wq, s, b = _weights(N, K, seed=N + M)
    g = torch.Generator(device="cuda")
    g.manual_seed(M)
    x = torch.randn(M, K, generator=g, device="cuda").half()
    logits = torch.empty(M, N, dtype=torch.float16, device="cuda")
    idx = qw_b200.quantized_matmul_argmax(x, wq, s, b, logits=logits)
    idx_nolog = qw_b200.quantized_matmul_argmax(x, wq, s, b)
    ref = qw_b200.quantized_matmul(x, wq, s, b)
    torch.cuda.synchronize()
    ref_np = ref.cpu().numpy()
    np.testing.assert_array_equal(logits.cpu().numpy().view(np.uint16), ref_np.view(np.uint16))
    expect = ref_np.astype(np.float32).argmax(axis=1)
    np.testing.assert_array_equal(idx.cpu().numpy(), expect)
    np.testing.assert_array_equal(idx_nolog.cpu().numpy(), expect)


def test_argmax_prefill_sized(cuda_dev):
    M, N, K = 40, 4096, 1024
    wq, s, b = _weights(N, K, seed=3)
    x = torch.randn(M, K, device="cuda").half()
    logits = torch.empty(M, N, dtype=torch.float16, device="cuda")
    idx = qw_b200.quantized_matmul_argmax(x, wq, s, b, logits=logits)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(idx.cpu().numpy(), logits.float().cpu().numpy().argmax(axis=1))
    with pytest.raises(_lib.QwError) as e:
        qw_b200.quantized_matmul_argmax(x, wq, s, b)
    assert e.value.code == _lib.QW_EINVAL


def test_ties_take_the_lowest_index(cuda_dev):
    N, K = 3000, 512
    wq = torch.full((N, K // 8), 0x12345678, dtype=torch.int32, device="cuda")  # every row identical
    s = torch.full((N, K // 64), 0.01, dtype=torch.float16, device="cuda")
    b = torch.full((N, K // 64), -0.05, dtype=torch.float16, device="cuda")
    x = torch.randn(3, K, device="cuda").half()
    idx = qw_b200.quantized_matmul_argmax(x, wq, s, b)
    torch.cuda.synchronize()
    assert idx.tolist() == [0, 0, 0]


def test_chosen_logit_is_the_oracle_max(cuda_dev):
    N, K, M = 2000, 1024, 2
    wq_np, s_np, b_np = oracle.quantize(synth.weight_fp16(N, K, seed=5))
    x = synth.activations(M, K, seed=5)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    idx = qw_b200.quantized_matmul_argmax(dev(x), dev(wq_np.view(np.int32)), dev(s_np), dev(b_np))
    torch.cuda.synchronize()
    _, y_ref = oracle.quantized_matmul(x, wq_np, s_np, b_np, want_f32=True)
    rms = np.sqrt(np.mean(y_ref.astype(np.float64) ** 2))
    for m, i in enumerate(idx.cpu().numpy()):
        assert abs(y_ref[m, i] - y_ref[m].max()) <= TOL * rms


@pytest.fixture(autouse=True)
def _clean_status(cuda_dev):
    yield
    assert qw_b200.device_status(0) == 0, "a kernel gave up on a bounded wait"
