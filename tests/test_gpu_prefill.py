"""GPU parity of the prefill path (M >= 17: tcgen05 MMA on dequantized tiles).

Against the CPU oracle at sizes it finishes quickly, and at the BASELINE's
prefill size (M=2048) against a plain fp32 torch matmul of the weights
dequantized by qw_dequantize (itself bit-exact with the oracle, see
test_gpu_parity.py).  Tolerance: max |y - y_ref| <= 1e-2 * rms(y_ref).
"""
import numpy as np
import pytest
import torch

import oracle
import qw_b200
from qw_b200 import synth
from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu


def dev_u32(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).cuda()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(autouse=True)
def _clean_status(cuda_dev):
    yield
    assert qw_b200.device_status(0) == 0, "a kernel gave up on a bounded wait"


# M <= 32 runs the 32-token tile (17, 24, 32), above it the 256-token tile
@pytest.mark.parametrize("M,N,K", [(17, 128, 64), (24, 1000, 5120), (32, 384, 1024), (33, 384, 1024),
                                   (64, 256, 512), (256, 384, 1024), (300, 200, 576),
                                   (40, 1000, 2048), (513, 136, 5120)])
def test_prefill_vs_oracle(M, N, K):
    w = synth.weight_fp16(N, K, seed=M + N)
    wq, s, b = oracle.quantize(w)
    x = synth.activations(M, K, seed=M)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    y = qw_b200.quantized_matmul(dev(x), dev_u32(wq), dev(s), dev(b))
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), y_ref) <= TOL
    # fp32 output: the path multiplies the bit-exact fp16 dequantized weights
    # (qw_dequantize's), so it matches their float64 product closely.
    y32 = qw_b200.quantized_matmul(dev(x), dev_u32(wq), dev(s), dev(b), out_dtype=torch.float32)
    torch.cuda.synchronize()
    y_deq = x.astype(np.float64) @ oracle.dequantize(wq, s, b).astype(np.float64).T
    assert rel_err(y32.cpu().numpy(), y_deq) <= 1e-4


def _torch_ref(x, wq, s, b):
    wd = qw_b200.dequantize(wq, s, b)  # bit-exact fp16 weights
    return (x.float() @ wd.float().t())


@pytest.mark.parametrize("N,K", [(17408, 5120), (5120, 17408), (8192, 5120)])
def test_prefill_full_size_vs_torch(N, K):
    """BASELINE prefill config: M=2048 tokens over the stack's shapes."""
    g = torch.Generator(device="cuda")
    g.manual_seed(N + K)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).half()
    wq, s, b = qw_b200.quantize_weights(w)
    x = torch.randn(2048, K, generator=g, device="cuda").half()
    y = qw_b200.quantized_matmul(x, wq, s, b)
    y_ref = _torch_ref(x, wq, s, b)
    torch.cuda.synchronize()
    err = (y.float() - y_ref).abs().max().item() / y_ref.pow(2).mean().sqrt().item()
    assert err <= TOL


def test_prefill_deterministic():
    N, K, M = 1024, 2048, 700
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).half()
    wq, s, b = qw_b200.quantize_weights(w)
    x = torch.randn(M, K, generator=g, device="cuda").half()
    y1 = qw_b200.quantized_matmul(x, wq, s, b, out_dtype=torch.float32)
    y2 = qw_b200.quantized_matmul(x, wq, s, b, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)


def test_prefill_extreme_scales_take_exact_path():
    """Scales below 2^-10 or above 63 use the per-element path; results still match."""
    N, K, M = 256, 512, 64
    rng = np.random.default_rng(3)
    wq = rng.integers(0, 2 ** 32, size=(N, K // 8), dtype=np.uint64).astype(np.uint32)
    s = np.where(rng.random((N, K // 64)) < 0.5, 1e-4, 80.0).astype(np.float16)
    b = (rng.standard_normal((N, K // 64)) * 0.01).astype(np.float16)
    x = (synth.activations(M, K, seed=3) * np.float16(0.01)).astype(np.float16)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    y32 = qw_b200.quantized_matmul(dev(x), dev_u32(wq), dev(s), dev(b), out_dtype=torch.float32)
    torch.cuda.synchronize()
    # the prefill path multiplies fp16-rounded weights: compare against them
    wd = oracle.dequantize(wq, s, b).astype(np.float64)
    y_deq = x.astype(np.float64) @ wd.T
    assert rel_err(y32.cpu().numpy(), y_deq) <= 1e-4
    assert rel_err(y32.cpu().numpy(), y_ref) <= TOL
