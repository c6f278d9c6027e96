"""GPU parity: libqwqmm.so (through its C ABI) against the CPU oracle.

Bars: quantize and dequantize bit-exact; matmul outputs within
max|y - y_ref| <= 1e-2 * rms(y_ref) (TOL), fp32 outputs within 1e-3.
"""
import numpy as np
import pytest
import torch

import oracle
import qw_b200
from qw_b200 import synth
from tests.conftest import TOL, golden_cases, load_golden, rel_err

pytestmark = pytest.mark.gpu


def dev_u32(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).cuda()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.cpu().numpy()


def quantized(N, K, seed=0):
    w = synth.weight_fp16(N, K, seed=seed)
    return oracle.quantize(w)


def run_qmm(x, wq, s, b, out_dtype=torch.float16):
    y = qw_b200.quantized_matmul(dev(x), dev_u32(wq), dev(s), dev(b), out_dtype=out_dtype)
    torch.cuda.synchronize()
    return host(y)


@pytest.fixture(autouse=True)
def _clean_status(cuda_dev):
    yield
    assert qw_b200.device_status(0) == 0, "a kernel gave up on a bounded wait"


# ---------------------------------------------------------------- golden
@pytest.mark.parametrize("name", golden_cases())
def test_golden_quantize_bit_exact(name):
    from tests.golden.gen_golden import CASES
    M, N, K, seed = CASES[name]
    w = synth.weight_fp16(N, K, seed=seed, layer=0, tid=0)
    g = load_golden(name)
    wq, s, b = qw_b200.quantize_weights(dev(w))
    np.testing.assert_array_equal(host(wq).view(np.uint32), g["wq"])
    np.testing.assert_array_equal(host(s).view(np.uint16), g["scales"].view(np.uint16))
    np.testing.assert_array_equal(host(b).view(np.uint16), g["biases"].view(np.uint16))


@pytest.mark.parametrize("name", golden_cases())
@pytest.mark.parametrize("rounding,key", [(0, "deq_twice"), (1, "deq_once")])
def test_golden_dequantize_bit_exact(name, rounding, key):
    g = load_golden(name)
    d = qw_b200.dequantize(dev_u32(g["wq"]), dev(g["scales"]), dev(g["biases"]), rounding=rounding)
    np.testing.assert_array_equal(host(d).view(np.uint16), g[key].view(np.uint16))


@pytest.mark.parametrize("name", golden_cases())
def test_golden_matmul(name):
    g = load_golden(name)
    y = run_qmm(g["x"], g["wq"], g["scales"], g["biases"])
    assert rel_err(y, g["y32"]) <= TOL
    y32 = run_qmm(g["x"], g["wq"], g["scales"], g["biases"], out_dtype=torch.float32)
    if g["x"].shape[0] <= 16:
        assert rel_err(y32, g["y32"]) <= 1e-3
    else:
        # M >= 17 multiplies the fp16 dequantized weights (deq_twice, bit-exact
        # with qw_dequantize): compare against their float64 product.
        y_deq = g["x"].astype(np.float64) @ g["deq_twice"].astype(np.float64).T
        assert rel_err(y32, y_deq) <= 1e-4


# ------------------------------------------------------------- sweeps
@pytest.mark.parametrize("M", list(range(1, 17)))
def test_every_small_m(M):
    wq, s, b = quantized(384, 1024, seed=M)
    x = synth.activations(M, 1024, seed=M)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    assert rel_err(run_qmm(x, wq, s, b), y_ref) <= TOL


@pytest.mark.parametrize("N,K", [(1, 64), (129, 64), (130, 576), (1000, 2048), (17, 4160), (512, 5120)])
@pytest.mark.parametrize("M", [1, 3, 5, 16])
def test_ragged_shapes(M, N, K):
    wq, s, b = quantized(N, K, seed=N + K)
    x = synth.activations(M, K, seed=N)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    assert rel_err(run_qmm(x, wq, s, b), y_ref) <= TOL


@pytest.mark.parametrize("N,K", [(300, 2112), (5000, 2176), (4000, 3648)])
def test_one_token_wide_units_ragged(N, K):
    """One token on shapes where the host takes 16-group (1024-wide) units
    although K is not a multiple of 1024: a partial last chunk, scales and
    biases staged with plain loads, and a ragged last row tile."""
    wq, s, b = quantized(N, K, seed=N ^ K)
    x = synth.activations(1, K, seed=K)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    assert rel_err(run_qmm(x, wq, s, b), y_ref) <= TOL
    assert rel_err(run_qmm(x, wq, s, b, out_dtype=torch.float32), y_ref) <= 1e-3


@pytest.mark.parametrize("M", [1, 4, 16])
def test_single_config_full_size(M):
    """BASELINE config: W [17408, 5120] 4-bit group 64, x ~ N(0, 1)."""
    wq, s, b = quantized(17408, 5120, seed=0)
    x = synth.activations(M, 5120, seed=0)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    y = run_qmm(x, wq, s, b)
    assert rel_err(y, y_ref) <= TOL
    y32 = run_qmm(x, wq, s, b, out_dtype=torch.float32)
    assert rel_err(y32, y_ref) <= 1e-3


def test_single_config_against_both_weight_conventions():
    """BASELINE's single configuration (seed 0, M=1) against the oracle in
    both weight-formation conventions: fp32-formed s*q + b (the decode
    kernel's arithmetic) and the fp16 `dequantize` weights (MLX's op-by-op
    output dtype).  Both within the north-star bar.  The kernel's fp32
    accumulators lie within 1e-4 * rms of the fp32-formed oracle's."""
    wq, s, b = quantized(17408, 5120, seed=0)
    x = synth.activations(1, 5120, seed=0)
    _, y_f32w = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    _, y_f16w = oracle.quantized_matmul(x, wq, s, b, weights="f16", want_f32=True)
    y = run_qmm(x, wq, s, b)
    assert rel_err(y, y_f32w) <= TOL
    assert rel_err(y, y_f16w) <= TOL
    y32 = run_qmm(x, wq, s, b, out_dtype=torch.float32)
    assert rel_err(y32, y_f32w) <= 1e-4
    assert rel_err(y32, y_f16w) <= 4e-3


def test_sixteen_and_seventeen_rows_agree_on_shared_rows():
    """The same 16 rows of x through the decode kernel (M=16, fp32-formed
    weights) and, with one more row, through the tensor-core kernel (M=17,
    fp16 ROUND_TWICE weights): a verify batch that grows past 16 rows changes
    arithmetic, and the shared rows' outputs move by at most 5e-3 * rms
    (half the north-star bar; the oracle's two conventions differ by 2.8e-3
    * rms at this shape, plus the fp16 output rounding)."""
    wq, s, b = quantized(17408, 5120, seed=0)
    x17 = synth.activations(17, 5120, seed=3)
    y16 = run_qmm(x17[:16], wq, s, b)
    y17 = run_qmm(x17, wq, s, b)
    _, y_ref = oracle.quantized_matmul(x17[:16], wq, s, b, want_f32=True)
    assert rel_err(y16, y_ref) <= TOL
    assert rel_err(y17[:16], y_ref) <= TOL
    d = np.abs(y16.astype(np.float64) - y17[:16].astype(np.float64))
    assert d.max() <= 5e-3 * np.sqrt(np.mean(y_ref.astype(np.float64) ** 2))
    y32_16 = run_qmm(x17[:16], wq, s, b, out_dtype=torch.float32)
    y32_17 = run_qmm(x17, wq, s, b, out_dtype=torch.float32)
    assert rel_err(y32_16, y32_17[:16]) <= 4e-3


@pytest.mark.parametrize("lin", synth.layer_linears() + [synth.LM_HEAD], ids=lambda l: l.name)
def test_stack_shapes_m1(lin):
    wq, s, b = quantized(lin.N, lin.K, seed=lin.tid)
    x = synth.activations(1, lin.K, seed=lin.tid)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    assert rel_err(run_qmm(x, wq, s, b), y_ref) <= TOL


def test_deterministic_across_calls():
    wq, s, b = quantized(5120, 17408, seed=3)   # down-projection shape: tiles split across CTAs
    x = synth.activations(3, 17408, seed=3)
    y1 = run_qmm(x, wq, s, b, out_dtype=torch.float32)
    y2 = run_qmm(x, wq, s, b, out_dtype=torch.float32)
    np.testing.assert_array_equal(y1, y2)


def test_large_m_runs_in_blocks():
    wq, s, b = quantized(256, 1024, seed=9)
    x = synth.activations(40, 1024, seed=9)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    assert rel_err(run_qmm(x, wq, s, b), y_ref) <= TOL


def test_leading_batch_dims():
    wq, s, b = quantized(200, 512, seed=4)
    x = synth.activations(6, 512, seed=4).reshape(2, 3, 512)
    y = qw_b200.quantized_matmul(dev(x), dev_u32(wq), dev(s), dev(b))
    assert tuple(y.shape) == (2, 3, 200)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    assert rel_err(host(y), y_ref) <= TOL


@pytest.mark.parametrize("M", [1, 4, 16, 40])
def test_row_strided_x(M):
    """x as a column slice of a wider matrix (rows 1536 apart) gives the same
    y as the contiguous copy, on the skinny (M <= 16) and prefill paths."""
    wq, s, b = quantized(300, 1024, seed=M)
    wide = torch.from_numpy(synth.activations(M, 1536, seed=M)).cuda()
    xs = wide[:, 256:256 + 1024]
    assert M == 1 or not xs.is_contiguous()
    y_s = qw_b200.quantized_matmul(xs, dev_u32(wq), dev(s), dev(b), out_dtype=torch.float32)
    y_c = qw_b200.quantized_matmul(xs.contiguous(), dev_u32(wq), dev(s), dev(b), out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(y_s, y_c)


# -------------------------------------------------------------- edge codes
@pytest.mark.parametrize("fill", [0x00000000, 0xFFFFFFFF, 0x0F0F0F0F])
def test_constant_codes(fill):
    N, K = 300, 1536
    wq = np.full((N, K // 8), fill, dtype=np.uint32)
    rng = np.random.default_rng(fill & 0xFF)
    s = (rng.random((N, K // 64)) * 0.01).astype(np.float16)
    b = (-rng.random((N, K // 64)) * 0.05).astype(np.float16)
    x = synth.activations(2, K, seed=1)
    _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    assert rel_err(run_qmm(x, wq, s, b), y_ref) <= TOL


def test_empty_inputs():
    wq, s, b = quantized(64, 128)
    x = torch.empty(0, 128, dtype=torch.float16, device="cuda")
    y = qw_b200.quantized_matmul(x, dev_u32(wq), dev(s), dev(b))
    assert tuple(y.shape) == (0, 64)


# ------------------------------------------------------- linear forwards
def test_linear_forward_bias_and_global_scale():
    N, K = 320, 1024
    wq, s, b = quantized(N, K, seed=12)
    x = synth.activations(3, K, seed=12)
    bias = (np.random.default_rng(1).standard_normal(N) * 0.1).astype(np.float16)
    gs = np.array([0.75], dtype=np.float32)
    y_ref = oracle.quantized_matmul(x, wq, s, b)  # fp16 output of the qmm
    lin = qw_b200.QuantizedLinear(dev_u32(wq), dev(s), dev(b), bias=dev(bias))
    y = host(lin(dev(x)))
    assert rel_err(y, (y_ref + bias).astype(np.float32)) <= TOL
    lin_gs = qw_b200.QuantizedLinear(dev_u32(wq), dev(s), dev(b), bias=dev(bias), global_scale=dev(gs))
    y2 = host(lin_gs(dev(x)))
    expect = (y_ref.astype(np.float32) * gs[0]).astype(np.float16) + bias
    assert rel_err(y2, expect) <= TOL


def test_invalid_call_raises_with_message():
    wq, s, b = quantized(64, 128)
    # 2-bit codes: the packing matches (8 words of 16 codes per row) but the width is unsupported
    with pytest.raises(qw_b200._lib.QwError, match="bits=2"):
        qw_b200.quantized_matmul(dev(synth.activations(1, 128)), dev_u32(np.ascontiguousarray(wq[:, :8])),
                                 dev(s), dev(b), bits=2)


def test_split_tiles_across_changing_grids():
    """Launches whose grids differ in size share the per-stream scratch; the
    split-tile counters must survive every sequence of shapes."""
    shapes = [(136, 1024), (40, 576), (5120, 17408), (72, 1536), (1000, 2048), (40, 576)]
    mats = [quantized(N, K, seed=i) for i, (N, K) in enumerate(shapes)]
    for rep in range(2):
        for (N, K), (wq, s, b) in zip(shapes, mats):
            x = synth.activations(1, K, seed=rep)
            _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
            assert rel_err(run_qmm(x, wq, s, b), y_ref) <= TOL, (N, K, rep)


@pytest.mark.parametrize("P", [4, 8])
@pytest.mark.parametrize("M", [1, 4, 16])
def test_tensor_parallel_shard_shapes(P, M):
    """Every shard shape of the BASELINE stack at TP=4 and TP=8 on one GPU:
    column shards (q|k|v, gate|up halves, lm_head) and row shards (o, down)
    whose K (1536/768, 4352/2176) is not a multiple of 512, so the decode
    kernel stages their scales and biases with plain loads.  Row shards
    return fp32 partial sums, as the exchange consumes them."""
    from qw_b200 import tp
    for lin in synth.layer_linears() + [synth.LM_HEAD]:
        N, K = tp.shard_shape(lin, P)
        if lin.name == "gate_up":
            N //= 2  # one of the two halves the fused SwiGLU reads
        wq, s, b = quantized(N, K, seed=N + K + P)
        x = synth.activations(M, K, seed=P)
        _, y_ref = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
        if lin.row_parallel:
            assert rel_err(run_qmm(x, wq, s, b, out_dtype=torch.float32), y_ref) <= 1e-3, (lin.name, N, K)
        else:
            assert rel_err(run_qmm(x, wq, s, b), y_ref) <= TOL, (lin.name, N, K)
