"""Fused SwiGLU input projections (qw_quantized_matmul_swiglu), the dense
quantized MLP (qw_swiglu_mlp), the standalone activation and the QuantizedMlp
module, against the oracle's op-by-op fp16 evaluation (two fp16 matmuls,
then sigmoid, gate * sigmoid and the product with up, each rounded to fp16).

The expected values follow the arithmetic of the kernel that runs (expected_mm):
fp32-formed weights on the decode kernel, as the oracle's matmul; the fp16
weights of dequantize on the tensor-core kernel (above 16 rows, and for the
8-bit and group-128 configurations), as its own parity tests use.

Tolerance (swiglu_close): |h - h_ref| <= 1e-2 rms(h_ref) + 2^-9 |h_ref| per
element.  The first term is the north-star output tolerance, which bounds
the fp32 accumulation error of gate and up; the second allows two fp16 ulps
of the value itself, because h is a product of two roughly Gaussian
factors: its tail reaches 30-40 rms, where one ulp of gate or up (or of h)
moved by a different summation order is already 1-2% of rms(h).  gate and
up are fp32 sums formed in another order than the oracle's (the decode
kernel folds each group as s * (d - Z) + b * X around an exact 1024
offset), so outputs are not bit-identical.  The standalone activation, fed
fp16 gate and up, is checked to one ulp."""
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


def dev_u32(a):
    return dev(np.ascontiguousarray(a).view(np.int32))


def proj(N, K, seed, gs=64, bits=4):
    return oracle.quantize(synth.weight_fp16(N, K, seed=seed), group_size=gs, bits=bits)


def on_dev(p):
    wq, s, b = p
    return dev_u32(wq), dev(s), dev(b)


def expected_mm(x, p, gs=64, bits=4):
    """The oracle's fp16 output of the kernel that runs this call: the decode
    kernel (at most 16 rows) forms each weight in fp32; the tensor-core
    kernel multiplies the fp16 weights of dequantize (rounding twice) with
    fp32 sums."""
    x = np.asarray(x, np.float16)
    if x.shape[0] <= 16:
        return oracle.quantized_matmul(x, *p, group_size=gs, bits=bits)
    w = oracle.dequantize(*p, group_size=gs, bits=bits).astype(np.float64)
    return (x.astype(np.float64) @ w.T).astype(np.float16)


def expected_h(x, gate, up, gs=64, bits=4):
    return oracle.swiglu(expected_mm(x, gate, gs, bits), expected_mm(x, up, gs, bits))


def swiglu_close(h, h_ref):
    h = np.asarray(h, np.float64)
    h_ref = np.asarray(h_ref, np.float64)
    if not h_ref.size:
        return True
    rms = np.sqrt(np.mean(h_ref ** 2))
    return bool(np.all(np.abs(h - h_ref) <= TOL * rms + 2.0 ** -9 * np.abs(h_ref)))


def identical_frac(a, b):
    a = np.asarray(a, np.float16).view(np.uint16)
    b = np.asarray(b, np.float16).view(np.uint16)
    return float(np.mean(a == b)) if a.size else 1.0


# (I, K): ragged I (not a multiple of the 64-row tile), K not a multiple of
# 512 (scales staged without TMA), cluster split-K (few tiles) and stream-K
# with split tiles (the model's 17408 x 5120 gate/up, 272 tiles).
SHAPES = [(200, 512), (64, 576), (1000, 2048), (2176, 5120), (17408, 5120)]


@pytest.mark.parametrize("I,K", SHAPES)
@pytest.mark.parametrize("M", [1, 3, 8, 16, 17, 300])
def test_swiglu_projection_vs_oracle(cuda_dev, I, K, M):
    if I == 17408 and M > 17:
        pytest.skip("covered at M <= 17; the oracle takes long at this size")
    gate, up = proj(I, K, seed=I + 1), proj(I, K, seed=I + 2)
    x = synth.activations(M, K, seed=M)
    h_ref = expected_h(x, gate, up)
    h = qw_b200.quantized_matmul_swiglu(dev(x), *on_dev(gate), *on_dev(up))
    torch.cuda.synchronize()
    h = h.cpu().numpy()
    assert h.shape == (M, I)
    assert np.isfinite(h.astype(np.float32)).all()
    assert swiglu_close(h, h_ref), rel_err(h, h_ref)


def test_fused_checkpoint_halves(cuda_dev):
    """Gate and up stored as one [2I] projection (fuse_mlp_input_projections)
    pass as two row views of the same buffers."""
    I, K, M = 328, 1024, 4
    wq, s, b = proj(2 * I, K, seed=5)
    x = synth.activations(M, K, seed=6)
    gate = (wq[:I], s[:I], b[:I])
    up = (wq[I:], s[I:], b[I:])
    h_ref = expected_h(x, gate, up)
    W, S, B = dev_u32(wq), dev(s), dev(b)
    for m in (M, 40):
        xm = synth.activations(m, K, seed=m)
        ref = expected_h(xm, gate, up)
        h = qw_b200.quantized_matmul_swiglu(dev(xm), W[:I], S[:I], B[:I], W[I:], S[I:], B[I:])
        torch.cuda.synchronize()
        assert swiglu_close(h.cpu().numpy(), ref)
    mlp = qw_b200.QuantizedMlp.from_fused(qw_b200.QuantizedLinear(W, S, B), I, down=None)
    assert mlp.fused
    h2 = mlp.forward_hidden(dev(x))
    torch.cuda.synchronize()
    assert swiglu_close(h2.cpu().numpy(), h_ref)


@pytest.mark.parametrize("bits,gs", [(4, 128), (8, 64), (8, 128)])
@pytest.mark.parametrize("M", [1, 9, 40])
def test_swiglu_other_configs(cuda_dev, bits, gs, M):
    """The other quantization configurations through both kernels' SwiGLU
    epilogues (decode kernel up to 16 rows, tensor-core kernel above)."""
    I, K = 200, 1536
    gate, up = proj(I, K, seed=11, gs=gs, bits=bits), proj(I, K, seed=12, gs=gs, bits=bits)
    x = synth.activations(M, K, seed=13)
    h_ref = expected_h(x, gate, up, gs, bits)
    h = qw_b200.quantized_matmul_swiglu(dev(x), *on_dev(gate), *on_dev(up), group_size=gs, bits=bits)
    torch.cuda.synchronize()
    assert swiglu_close(h.cpu().numpy(), h_ref)


def test_activation_kernel_vs_oracle(cuda_dev):
    """The standalone activation on fp16 inputs: the only difference from the
    oracle is the float32 sigmoid's last bits, which fp16 rounding hides on
    nearly every element."""
    rng = np.random.default_rng(0)
    g = (rng.standard_normal((7, 1001)) * 4).astype(np.float16)
    u = rng.standard_normal((7, 1001)).astype(np.float16)
    g[0, :6] = [-65504, -100, -20, 0, 20, 65504]
    ref = oracle.swiglu(g, u)
    out = qw_b200.compiled_swiglu_activation(dev(g), dev(u))
    torch.cuda.synchronize()
    out = out.cpu().numpy()
    assert identical_frac(out, ref) >= 0.999
    diff = np.abs(out.view(np.uint16).astype(np.int32) - ref.view(np.uint16).astype(np.int32))
    assert diff.max() <= 1  # at most one fp16 ulp apart
    assert out[0, 0] == 0 and out[0, 1] == 0 and out[0, 3] == 0


@pytest.mark.parametrize("M", [1, 16, 64])
def test_swiglu_mlp_vs_oracle(cuda_dev, M):
    """down(silu(gate(x)) * up(x)) end to end (compiled_moe_expert_forward)."""
    H, I = 512, 1408
    gate, up, down = proj(I, H, seed=21), proj(I, H, seed=22), proj(H, I, seed=23)
    x = synth.activations(M, H, seed=24)
    y_ref = expected_mm(expected_h(x, gate, up), down)
    y = qw_b200.swiglu_mlp(dev(x), *on_dev(gate), *on_dev(up), *on_dev(down))
    mlp = qw_b200.QuantizedMlp(qw_b200.QuantizedLinear(*on_dev(gate)), qw_b200.QuantizedLinear(*on_dev(up)),
                               qw_b200.QuantizedLinear(*on_dev(down)))
    y2 = mlp(dev(x))
    torch.cuda.synchronize()
    assert y.shape == (M, H)
    assert rel_err(y.cpu().numpy(), y_ref) <= TOL
    assert rel_err(y2.cpu().numpy(), y_ref) <= TOL


def test_separate_arm_matches_fused(cuda_dev):
    """A gate and up with different quantization cannot fuse (the reference's
    Separate arm): two matmuls and the activation kernel, same result."""
    I, K, M = 256, 1024, 5
    g4 = proj(I, K, seed=31)
    u8 = proj(I, K, seed=32, bits=8)
    x = synth.activations(M, K, seed=33)
    ref = oracle.swiglu(expected_mm(x, g4), expected_mm(x, u8, bits=8))
    down = qw_b200.QuantizedLinear(*on_dev(proj(64, I, seed=34)))
    mlp = qw_b200.QuantizedMlp(qw_b200.QuantizedLinear(*on_dev(g4)),
                               qw_b200.QuantizedLinear(*on_dev(u8), bits=8), down)
    assert not mlp.fused
    h = mlp.forward_hidden(dev(x))
    torch.cuda.synchronize()
    assert swiglu_close(h.cpu().numpy(), ref)


def test_swiglu_errors(cuda_dev):
    gate, up = proj(128, 512, seed=41), proj(64, 512, seed=42)
    x = dev(synth.activations(1, 512))
    with pytest.raises(_lib.QwError, match="same shape"):
        qw_b200.quantized_matmul_swiglu(x, *on_dev(gate), *on_dev(up))
    g, s, b = on_dev(gate)
    with pytest.raises(_lib.QwError, match="requires biases"):
        qw_b200.quantized_matmul_swiglu(x, g, s, b, g, s, None)
    with pytest.raises(_lib.QwError, match="same shape"):
        qw_b200.compiled_swiglu_activation(dev(np.zeros((2, 3), np.float16)), dev(np.zeros((3, 2), np.float16)))


def test_swiglu_empty(cuda_dev):
    gate = proj(128, 512, seed=51)
    x = torch.empty(0, 512, dtype=torch.float16, device="cuda")
    h = qw_b200.quantized_matmul_swiglu(x, *on_dev(gate), *on_dev(gate))
    assert h.shape == (0, 128)
