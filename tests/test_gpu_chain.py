"""qw_quantized_matmul_chain: dependent matmuls in one cooperative launch.

Each chain is checked against the same matmuls issued one by one through
qw_quantized_matmul (the reduction order differs, so within the output
tolerance), and a short chain against the CPU oracle.  Shapes cover row-tile
counts below and above the SM count, K not a multiple of 512 (scales and
biases staged without TMA), ragged N, fp32 outputs, chains longer than one
launch takes, and a prefill-sized chain (one launch per matmul).
Tolerance: max |y - y_ref| <= 1e-2 * rms(y_ref)."""
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


def _run_chain(M, dims, seed=0, f32_every=0):
    """dims = [K0, N0(=K1), N1, ...]: op i maps dims[i] -> dims[i+1], chained."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x0 = torch.randn(M, dims[0], generator=g, device="cuda").half()
    ws = [_weights(dims[i + 1], dims[i], seed=seed * 100 + i) for i in range(len(dims) - 1)]
    ys = []
    ops = []
    x = x0
    for i, (wq, s, b) in enumerate(ws):
        y = torch.full((M, dims[i + 1]), float("nan"), device="cuda", dtype=torch.float16)
        ops.append((x, wq, s, b, y))
        ys.append(y)
        x = y
    qw_b200.quantized_matmul_chain(ops)
    # reference: one qw_quantized_matmul per op, on the chain's own inputs
    refs = [qw_b200.quantized_matmul(op[0], op[1], op[2], op[3]) for op in ops]
    torch.cuda.synchronize()
    return x0, ws, ys, refs


@pytest.mark.parametrize("M", [1, 4, 16])
def test_chain_matches_one_by_one(cuda_dev, M):
    dims = [5120, 8192, 6144, 5120, 17408, 5120]
    _, _, ys, refs = _run_chain(M, dims, seed=M)
    for i, (y, r) in enumerate(zip(ys, refs)):
        y_np, r_np = y.float().cpu().numpy(), r.float().cpu().numpy()
        assert np.isfinite(y_np).all(), i
        assert rel_err(y_np, r_np) <= TOL, i


@pytest.mark.parametrize("M", [1, 5])
def test_chain_ragged_and_small_shapes(cuda_dev, M):
    # K % 512 != 0 (every op), few row tiles, and a last N that is not a
    # multiple of the 128-row tile (an op's N is the next op's K, a multiple of 64)
    dims = [576, 192, 1088, 64, 4160, 1000]
    _, _, ys, refs = _run_chain(M, dims, seed=7 + M)
    for i, (y, r) in enumerate(zip(ys, refs)):
        assert rel_err(y.float().cpu().numpy(), r.float().cpu().numpy()) <= TOL, i


def test_chain_longer_than_one_launch(cuda_dev):
    dims = [1024] * 31 + [512]  # 31 ops, more than one launch's 24
    _, _, ys, refs = _run_chain(1, dims, seed=3)
    for i, (y, r) in enumerate(zip(ys, refs)):
        assert rel_err(y.float().cpu().numpy(), r.float().cpu().numpy()) <= TOL, i


def test_chain_vs_oracle(cuda_dev):
    M, dims = 2, [512, 384, 640, 256]
    x0, ws, ys, _ = _run_chain(M, dims, seed=11)
    x = x0.cpu().numpy()
    for i, (wq, s, b) in enumerate(ws):
        wq_np = wq.cpu().numpy().view(np.uint32)
        _, y32 = oracle.quantized_matmul(x, wq_np, s.cpu().numpy(), b.cpu().numpy(), want_f32=True)
        assert rel_err(ys[i].float().cpu().numpy(), y32) <= TOL, i
        x = ys[i].cpu().numpy()  # the next op reads the chain's fp16 output


def test_chain_fp32_outputs_and_prefill_sized(cuda_dev):
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    for M in (1, 64):
        x = torch.randn(M, 1024, generator=g, device="cuda").half()
        wq, s, b = _weights(2048, 1024, seed=21)
        y32 = torch.empty(M, 2048, device="cuda", dtype=torch.float32)
        qw_b200.quantized_matmul_chain([(x, wq, s, b, y32)])
        ref = qw_b200.quantized_matmul(x, wq, s, b, out_dtype=torch.float32)
        torch.cuda.synchronize()
        assert rel_err(y32.cpu().numpy(), ref.cpu().numpy()) <= TOL


def test_chain_rejects_mixed_rows(cuda_dev):
    wq, s, b = _weights(256, 512, seed=1)
    x1 = torch.zeros(1, 512, device="cuda", dtype=torch.float16)
    x2 = torch.zeros(2, 512, device="cuda", dtype=torch.float16)
    y1 = torch.empty(1, 256, device="cuda", dtype=torch.float16)
    y2 = torch.empty(2, 256, device="cuda", dtype=torch.float16)
    with pytest.raises(_lib.QwError) as e:
        qw_b200.quantized_matmul_chain([(x1, wq, s, b, y1), (x2, wq, s, b, y2)])
    assert e.value.code == _lib.QW_EINVAL
    assert "rows of x" in str(e.value)


@pytest.fixture(autouse=True)
def _clean_status(cuda_dev):
    yield
    assert qw_b200.device_status(0) == 0, "a kernel gave up on a bounded wait"
