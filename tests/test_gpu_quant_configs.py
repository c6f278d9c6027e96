"""The other quantization configurations of QW's per-tensor overrides:
8-bit codes and groups of 128 (4/128, 8/64, 8/128).  Quantize and dequantize
are bit-exact with the oracle; the matmul is within the output tolerance of
the oracle, and its fp32 output within 1e-4 of the product it forms: the
oracle's fp32-formed weights on the decode kernel (up to 16 rows), the
float64 product of the bit-exact dequantized weights on the tensor-core
kernel (more rows).  The decode kernel's 8-bit codes are also checked at the
model's shapes and at ragged edges (K not a multiple of its 512-wide chunk,
N not a multiple of its 128-row tile).  Entry points that only take 4-bit
codes say so."""
import functools

import numpy as np
import pytest
import torch

import oracle
import qw_b200
from qw_b200 import _lib, synth
from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu
CONFIGS = [(4, 128), (8, 64), (8, 128)]


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def dev_u32(a):
    return dev(np.ascontiguousarray(a).view(np.int32))


@pytest.mark.parametrize("bits,gs", CONFIGS)
def test_quantize_and_dequantize_bit_exact(cuda_dev, bits, gs):
    N, K = 300, 1536
    w = synth.weight_fp16(N, K, seed=bits * gs)
    wq, s, b = qw_b200.quantize_weights(dev(w), group_size=gs, bits=bits)
    rq, rs, rb = oracle.quantize(w, group_size=gs, bits=bits)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(wq.cpu().numpy().view(np.uint32), rq)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), rs.view(np.uint16))
    np.testing.assert_array_equal(b.cpu().numpy().view(np.uint16), rb.view(np.uint16))
    for rounding in (0, 1):
        d = qw_b200.dequantize(dev_u32(rq), dev(rs), dev(rb), group_size=gs, bits=bits, rounding=rounding)
        ref = oracle.dequantize(rq, rs, rb, group_size=gs, bits=bits, rounding=rounding)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(d.cpu().numpy().view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("bits,gs", CONFIGS)
@pytest.mark.parametrize("M", [1, 5, 16, 32, 33, 40, 300])
def test_matmul_vs_oracle(cuda_dev, bits, gs, M):
    N, K = 384, 1280 if gs == 64 else 1536
    wq, s, b = oracle.quantize(synth.weight_fp16(N, K, seed=M + bits), group_size=gs, bits=bits)
    x = synth.activations(M, K, seed=M)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, group_size=gs, bits=bits, want_f32=True)
    y = qw_b200.quantized_matmul(dev(x), dev_u32(wq), dev(s), dev(b), group_size=gs, bits=bits)
    y32 = qw_b200.quantized_matmul(dev(x), dev_u32(wq), dev(s), dev(b), group_size=gs, bits=bits,
                                   out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), y_ref) <= TOL
    if M <= 16:
        # the decode kernel forms each weight in fp32 as the oracle does
        assert rel_err(y32.cpu().numpy(), y_ref) <= 1e-4
    else:
        # the tensor-core kernel multiplies the bit-exact fp16 dequantized weights
        y_deq = x.astype(np.float64) @ oracle.dequantize(wq, s, b, group_size=gs, bits=bits).astype(np.float64).T
        assert rel_err(y32.cpu().numpy(), y_deq) <= 1e-4


@pytest.mark.parametrize("bits,gs", CONFIGS)
def test_extreme_scales_take_the_exact_path(cuda_dev, bits, gs):
    N, K, M = 256, 1024, 20
    rng = np.random.default_rng(bits)
    wq = rng.integers(0, 2 ** 32, size=(N, K * bits // 32), dtype=np.uint64).astype(np.uint32)
    s = np.where(rng.random((N, K // gs)) < 0.5, 1e-4, 80.0).astype(np.float16)
    b = (rng.standard_normal((N, K // gs)) * 0.01).astype(np.float16)
    x = (synth.activations(M, K, seed=3) * np.float16(0.01)).astype(np.float16)
    y32 = qw_b200.quantized_matmul(dev(x), dev_u32(wq), dev(s), dev(b), group_size=gs, bits=bits,
                                   out_dtype=torch.float32)
    torch.cuda.synchronize()
    wd = oracle.dequantize(wq, s, b, group_size=gs, bits=bits).astype(np.float64)
    assert rel_err(y32.cpu().numpy(), x.astype(np.float64) @ wd.T) <= 1e-4


def test_other_configs_in_chains_argmax_and_static_scratch(cuda_dev):
    N, K = 512, 1024
    wq, s, b = oracle.quantize(synth.weight_fp16(N, K, seed=8), group_size=64, bits=8)
    w_d, s_d, b_d = dev_u32(wq), dev(s), dev(b)
    x = dev(synth.activations(2, K, seed=8))
    y_chain = torch.empty(2, N, dtype=torch.float16, device="cuda")
    qw_b200.quantized_matmul_chain([(x, w_d, s_d, b_d, y_chain)], group_size=64, bits=8)
    y = qw_b200.quantized_matmul(x, w_d, s_d, b_d, group_size=64, bits=8)
    logits = torch.empty(2, N, dtype=torch.float16, device="cuda")
    idx = qw_b200.quantized_matmul_argmax(x, w_d, s_d, b_d, group_size=64, bits=8, logits=logits)
    torch.cuda.synchronize()
    assert torch.equal(y_chain, y)
    assert idx.tolist() == logits.float().cpu().numpy().argmax(axis=1).tolist()
    # up to 16 rows the greedy token needs no logits buffer (the decode
    # kernel's epilogue); more rows do
    idx2 = qw_b200.quantized_matmul_argmax(x, w_d, s_d, b_d, group_size=64, bits=8)
    assert idx2.tolist() == idx.tolist()
    x40 = dev(synth.activations(40, K, seed=9))
    with pytest.raises(_lib.QwError) as e:
        qw_b200.quantized_matmul_argmax(x40, w_d, s_d, b_d, group_size=64, bits=8)
    assert e.value.code == _lib.QW_EINVAL
    L = _lib.load()
    from qw_b200.ops import _arr, _mode, _stream
    y_static = torch.empty_like(y)
    rc = L.qw_quantized_matmul_static_scratch(_arr(x), _arr(w_d), _arr(s_d), _arr(b_d), 1, 64, 8, _mode("affine"),
                                              _arr(y_static), _stream(x))
    torch.cuda.synchronize()
    assert rc == _lib.QW_OK
    assert torch.equal(y_static, y)


@functools.lru_cache(maxsize=4)
def _weights8(N, K, gs):
    return oracle.quantize(synth.weight_fp16(N, K, seed=N + K), group_size=gs, bits=8)


@pytest.mark.parametrize("gs", [64, 128])
@pytest.mark.parametrize("N,K", [(1000, 2048), (5120, 17408), (17408, 5120), (300, 576), (130, 64)])
@pytest.mark.parametrize("M", [1, 3, 8, 9, 16])
def test_decode_kernel_8bit_shapes(cuda_dev, gs, N, K, M):
    """8-bit codes on the decode kernel: the projections of the model's MLP
    (split over clusters or stream-K, scales through TMA or staged), a row
    tile cut by N, and K of one group or with a partial last chunk."""
    if K % gs:
        pytest.skip("K is not a multiple of the group")
    wq, s, b = _weights8(N, K, gs)
    x = synth.activations(M, K, seed=K + M)
    y_ref, y32_ref = oracle.quantized_matmul(x, wq, s, b, group_size=gs, bits=8, want_f32=True)
    w_d, s_d, b_d = dev_u32(wq), dev(s), dev(b)
    y = qw_b200.quantized_matmul(dev(x), w_d, s_d, b_d, group_size=gs, bits=8)
    y32 = qw_b200.quantized_matmul(dev(x), w_d, s_d, b_d, group_size=gs, bits=8, out_dtype=torch.float32)
    idx = qw_b200.quantized_matmul_argmax(dev(x), w_d, s_d, b_d, group_size=gs, bits=8)
    torch.cuda.synchronize()
    assert rel_err(y.cpu().numpy(), y32_ref) <= TOL
    assert rel_err(y32.cpu().numpy(), y32_ref) <= 1e-4
    yh = y.cpu().numpy()
    assert idx.tolist() == yh.astype(np.float32).argmax(axis=1).tolist()


@pytest.fixture(autouse=True)
def _clean_status(cuda_dev):
    yield
    assert qw_b200.device_status(0) == 0, "a kernel gave up on a bounded wait"
