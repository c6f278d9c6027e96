"""CPU tests of the oracle: hand-derived known answers, the reference's own
layout test restated, the committed golden fixtures, and agreement with the
independent numpy restatement.  No GPU."""
import numpy as np
import pytest

import oracle
from oracle import np_ref
from qw_b200 import synth
from tests.conftest import golden_cases, load_golden, rel_err


def f16(*v):
    return np.array(v, dtype=np.float16)


# ---------------------------------------------------------------- fp16 helpers
def test_f16_conversion_matches_numpy_on_every_pattern():
    L = oracle.lib()
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    ours = np.array([L.qwo_f16_to_f32(int(b)) for b in bits[::97]], dtype=np.float32)
    np.testing.assert_array_equal(np.isnan(ours), np.isnan(ref[::97]))
    ok = ~np.isnan(ref[::97])
    np.testing.assert_array_equal(ours[ok], ref[::97][ok])


def test_f32_to_f16_round_to_nearest_even():
    L = oracle.lib()
    rng = np.random.default_rng(7)
    vals = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * 10,
        rng.standard_normal(1000).astype(np.float32) * 1e-6,   # subnormal range
        np.array([65504, 65519.99, 65520, 1e9, -1e9, 2.0 ** -25, 2.0 ** -24, 3 * 2.0 ** -26, 0.0, -0.0],
                 dtype=np.float32),
    ])
    ours = np.array([L.qwo_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    with np.errstate(over="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    np.testing.assert_array_equal(ours, ref)
    # float64 path: compare against numpy's direct double -> half conversion
    d = rng.standard_normal(3000) * 3.0
    ours64 = np.array([L.qwo_f64_to_f16(float(v)) for v in d], dtype=np.uint16)
    np.testing.assert_array_equal(ours64, d.astype(np.float16).view(np.uint16))


# ------------------------------------------------------------ known answers
def test_nibble_order_known_answer():
    """Element k of a row is bits 4*(k%8).. of word k/8, low nibble first."""
    K = 64
    words = np.array([[0x76543210, 0xFEDCBA98] * 4], dtype=np.uint32)  # codes 0..15, 0..15, ...
    s = f16(0.5).reshape(1, 1)
    b = f16(-1.0).reshape(1, 1)
    deq = oracle.dequantize(words, s, b)
    expect = (np.tile(np.arange(16), 4) * 0.5 - 1.0).astype(np.float16).reshape(1, K)
    np.testing.assert_array_equal(deq, expect)
    # x = e_k picks out column k exactly
    for k in (0, 1, 7, 8, 15, 63):
        x = np.zeros((1, K), dtype=np.float16)
        x[0, k] = 1.0
        y = oracle.quantized_matmul(x, words, s, b)
        assert float(y[0, 0]) == float(expect[0, k])


def test_all_zero_and_all_fifteen_codes():
    K, N = 128, 3
    s = np.full((N, K // 64), 0.25, dtype=np.float16)
    b = np.full((N, K // 64), 0.125, dtype=np.float16)
    zeros = np.zeros((N, K // 8), dtype=np.uint32)
    full = np.full((N, K // 8), 0xFFFFFFFF, dtype=np.uint32)
    np.testing.assert_array_equal(oracle.dequantize(zeros, s, b), np.full((N, K), 0.125, np.float16))
    np.testing.assert_array_equal(oracle.dequantize(full, s, b), np.full((N, K), 3.875, np.float16))
    x = np.ones((2, K), dtype=np.float16)
    np.testing.assert_array_equal(oracle.quantized_matmul(x, full, s, b), np.full((2, N), 496.0, np.float16))


def test_roundings_differ_only_where_expected():
    """Rounded-once and rounded-twice dequantisation agree on exactly
    representable cases and otherwise differ by at most the first rounding
    (half an ulp of s*q) plus one ulp of the result."""
    rng = np.random.default_rng(3)
    N, K = 64, 256
    wq = rng.integers(0, 2 ** 32, size=(N, K // 8), dtype=np.uint64).astype(np.uint32)
    s = (rng.random((N, K // 64)) * 0.01).astype(np.float16)
    b = (-rng.random((N, K // 64)) * 0.08).astype(np.float16)
    d0 = oracle.dequantize(wq, s, b, rounding=oracle.ROUND_TWICE).astype(np.float64)
    d1 = oracle.dequantize(wq, s, b, rounding=oracle.ROUND_ONCE).astype(np.float64)
    sq = np.repeat(s, 64, axis=1).astype(np.float64) * np_ref.unpack(wq).astype(np.float64)
    bound = 0.5 * np.spacing(np.abs(sq).astype(np.float16)).astype(np.float64) + \
        np.spacing(np.abs(d1).astype(np.float16)).astype(np.float64)
    assert np.all(np.abs(d0 - d1) <= bound * 1.0001)
    assert np.mean(d0 != d1) > 0.05  # the two conventions really differ
    pow2 = np.full_like(s, 0.25)
    np.testing.assert_array_equal(oracle.dequantize(wq, pow2, f16(0).reshape(1, 1).repeat(N, 0).repeat(K // 64, 1)),
                                  oracle.dequantize(wq, pow2, np.zeros_like(b), rounding=oracle.ROUND_ONCE))


def test_dequantize_commutes_with_output_axis_slice():
    """The reference's one deterministic dequantize test
    (crates/mlxcel-core/src/ffi_tests.rs:3792-3850), restated with its hand-made
    word patterns: dequantize(slice(w)) == slice(dequantize(w)) bit for bit.
    The reference uses group 32 and f32 scales; here group 64 / fp16 scales,
    which the same property covers."""
    experts, rows, K = 2, 8, 128
    packed = K // 8
    groups = K // 64
    w = np.zeros((experts * rows, packed), dtype=np.uint32)
    s = np.zeros((experts * rows, groups), dtype=np.float16)
    b = np.zeros((experts * rows, groups), dtype=np.float16)
    for e in range(experts):
        for r in range(rows):
            for c in range(packed):
                w[e * rows + r, c] = (0x12345678 + e * 131 + r * 17 + c) & 0xFFFFFFFF
            for g in range(groups):
                s[e * rows + r, g] = 0.05 + 0.01 * e + 0.001 * r + 0.0003 * g
                b[e * rows + r, g] = -0.2 + 0.02 * e - 0.003 * r + 0.0007 * g
    full = oracle.dequantize(w, s, b)
    half = rows // 2
    for e in range(experts):
        for lo, hi in ((0, half), (half, rows)):
            sl = slice(e * rows + lo, e * rows + hi)
            part = oracle.dequantize(np.ascontiguousarray(w[sl]), np.ascontiguousarray(s[sl]),
                                     np.ascontiguousarray(b[sl]))
            np.testing.assert_array_equal(part.view(np.uint16), full[sl].view(np.uint16))


def _reference_layout_case():
    """The exact inputs of crates/mlxcel-core/src/ffi_tests.rs:3792-3850:
    2 experts x 8 rows x 64 inputs, 4 bits, group 32, word (e, r, c) =
    0x12345678 + 131e + 17r + c, float32 scales 0.05 + 0.01e + 0.001r +
    0.0003g and biases -0.2 + 0.02e - 0.003r + 0.0007g (each formed in
    float32 as the reference's Rust expressions are)."""
    experts, rows, K, gs = 2, 8, 64, 32
    packed, groups = K * 4 // 32, K // gs
    w = np.zeros((experts, rows, packed), dtype=np.uint32)
    s = np.zeros((experts, rows, groups), dtype=np.float32)
    b = np.zeros((experts, rows, groups), dtype=np.float32)
    f = np.float32
    for e in range(experts):
        for r in range(rows):
            for c in range(packed):
                w[e, r, c] = (0x12345678 + e * 131 + r * 17 + c) & 0xFFFFFFFF
            for g in range(groups):
                s[e, r, g] = f(0.05) + f(0.01) * f(e) + f(0.001) * f(r) + f(0.0003) * f(g)
                b[e, r, g] = f(-0.2) + f(0.02) * f(e) - f(0.003) * f(r) + f(0.0007) * f(g)
    return w, s, b, gs


@pytest.mark.parametrize("rounding", [oracle.ROUND_TWICE, oracle.ROUND_ONCE])
def test_reference_layout_case_exact_inputs(rounding):
    """The reference's deterministic dequantize test on its own inputs (group
    32, float32 scales and biases, [2, 8, 64]): dequantizing each half of the
    row axis equals the same half of the whole tensor's dequantization, bit
    for bit; and every element is the stated float32 sequence (s*q then + b,
    or one fused rounding), checked against numpy."""
    w, s, b, gs = _reference_layout_case()
    E, R, _ = w.shape
    full = oracle.dequantize_f32(w.reshape(E * R, -1), s.reshape(E * R, -1), b.reshape(E * R, -1),
                                 group_size=gs, rounding=rounding).reshape(E, R, -1)
    assert full.shape == (2, 8, 64) and full.dtype == np.float32
    half = R // 2
    for lo, hi in ((0, half), (half, R)):
        part = oracle.dequantize_f32(np.ascontiguousarray(w[:, lo:hi]).reshape(E * (hi - lo), -1),
                                     np.ascontiguousarray(s[:, lo:hi]).reshape(E * (hi - lo), -1),
                                     np.ascontiguousarray(b[:, lo:hi]).reshape(E * (hi - lo), -1),
                                     group_size=gs, rounding=rounding).reshape(E, hi - lo, -1)
        assert part.tobytes() == np.ascontiguousarray(full[:, lo:hi]).tobytes()
    # element values: nibble k of the row at bits 4*(k % 8) of word k // 8
    k = np.arange(64)
    q = ((w[..., k // 8] >> (4 * (k % 8)).astype(np.uint32)) & 0xF).astype(np.float32)
    sg, bg = np.repeat(s, gs, axis=-1), np.repeat(b, gs, axis=-1)
    if rounding == oracle.ROUND_TWICE:
        want = (sg * q).astype(np.float32) + bg
    else:
        want = (sg.astype(np.float64) * q + bg).astype(np.float32)  # s*q is exact in float64
    np.testing.assert_array_equal(full.view(np.uint32), want.astype(np.float32).view(np.uint32))


def test_reference_layout_case_in_fp16():
    """The same words, scales and biases cast to fp16 (the checkpoint's scale
    dtype): the fp16 dequantization at group 32 commutes with the row slice
    and matches the numpy restatement bit for bit."""
    w, s, b, gs = _reference_layout_case()
    E, R, P = w.shape
    w2, s2, b2 = w.reshape(E * R, P), s.reshape(E * R, -1).astype(np.float16), b.reshape(E * R, -1).astype(np.float16)
    full = oracle.dequantize(w2, s2, b2, group_size=gs)
    np.testing.assert_array_equal(full.view(np.uint16), np_ref.dequantize(w2, s2, b2, group_size=gs).view(np.uint16))
    for e in range(E):
        for lo, hi in ((0, R // 2), (R // 2, R)):
            sl = slice(e * R + lo, e * R + hi)
            part = oracle.dequantize(np.ascontiguousarray(w2[sl]), np.ascontiguousarray(s2[sl]),
                                     np.ascontiguousarray(b2[sl]), group_size=gs)
            np.testing.assert_array_equal(part.view(np.uint16), full[sl].view(np.uint16))


def test_weight_formation_modes_are_their_stated_sequences():
    """weights="f16" multiplies the ROUND_TWICE fp16 weights, summing fp32
    products in ascending k; quantized_matmul_f16acc rounds every product and
    every partial sum to fp16.  Both checked against plain Python loops."""
    w = synth.weight_fp16(9, 192, seed=41)
    wq, s, b = oracle.quantize(w)
    x = synth.activations(3, 192, seed=42)
    w16 = oracle.dequantize(wq, s, b)
    y16w = oracle.quantized_matmul(x, wq, s, b, weights="f16")
    y16acc = oracle.quantized_matmul_f16acc(x, wq, s, b)
    for m in range(3):
        for n in range(9):
            acc = np.float32(0)
            acc16 = np.float16(0)
            for k in range(192):
                p = np.float32(x[m, k]) * np.float32(w16[n, k])
                acc = np.float32(acc + p)
                acc16 = np.float16(np.float32(acc16) + np.float32(np.float16(p)))
            assert y16w[m, n].view(np.uint16) == np.float16(acc).view(np.uint16)
            assert y16acc[m, n].view(np.uint16) == acc16.view(np.uint16)


def test_weight_formation_convention_is_inside_the_bar():
    """How far the two float32-accumulating conventions lie apart at
    BASELINE's single configuration (x [1, 5120], W [17408, 5120], seed 0):
    fp32-formed weights (the oracle's default) against the fp16 `dequantize`
    weights (MLX's op-by-op dtype).  Measured 2.8e-3 * rms; the north-star
    bar is 1e-2 * rms, so either convention passes against the other.
    Accumulating in fp16 instead (quantized_matmul_f16acc, every product
    and partial sum rounded) lands 8.4e-2 * rms away at this K, far outside
    the bar, which is why the oracle pins float32 accumulation as the north
    star states; here that is shown on 1024 of the rows."""
    N, K = 17408, 5120
    w = synth.weight_fp16(N, K, seed=0)
    wq, s, b = oracle.quantize(w)
    x = synth.activations(1, K, seed=0)
    _, y32 = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    y16w = oracle.quantized_matmul(x, wq, s, b, weights="f16")
    assert rel_err(y16w, y32) <= 4e-3
    rows = slice(0, 1024)
    y16acc = oracle.quantized_matmul_f16acc(x, wq[rows], s[rows], b[rows])
    assert rel_err(y16acc, y32[:, rows]) > 2e-2


def test_packing_invariant_is_enforced():
    """packed_in * 32 == bits * groups * group_size (layers.rs:1568-1570)."""
    with pytest.raises(ValueError):
        oracle.quantized_matmul(np.zeros((1, 128), np.float16), np.zeros((2, 8), np.uint32),
                                np.zeros((2, 2), np.float16), np.zeros((2, 2), np.float16))


# ------------------------------------------------------------- restatements
@pytest.mark.parametrize("bits,gs", [(8, 64), (4, 128), (8, 128)])
def test_restatements_agree_for_other_configs(bits, gs):
    """The 8-bit and group-128 configurations of the per-tensor overrides."""
    N, K = 40, 768
    w = synth.weight_fp16(N, K, seed=bits + gs)
    wq, s, b = oracle.quantize(w, group_size=gs, bits=bits)
    wq2, s2, b2 = np_ref.quantize(w, group_size=gs, bits=bits)
    np.testing.assert_array_equal(wq, wq2)
    np.testing.assert_array_equal(s.view(np.uint16), s2.view(np.uint16))
    np.testing.assert_array_equal(b.view(np.uint16), b2.view(np.uint16))
    for r, name in ((oracle.ROUND_TWICE, "twice"), (oracle.ROUND_ONCE, "once")):
        np.testing.assert_array_equal(
            oracle.dequantize(wq, s, b, group_size=gs, bits=bits, rounding=r).view(np.uint16),
            np_ref.dequantize(wq, s, b, group_size=gs, bits=bits, rounding=name).view(np.uint16))
    x = synth.activations(3, K, seed=2)
    _, y32 = oracle.quantized_matmul(x, wq, s, b, group_size=gs, bits=bits, want_f32=True)
    assert rel_err(y32, np_ref.quantized_matmul(x, wq, s, b, group_size=gs, bits=bits)) < 1e-5


def test_eight_bit_code_order_known_answer():
    """8-bit codes: element k of a row is byte k % 4 of word k / 4."""
    wq = np.array([[0x04030201, 0xFF00807F]], dtype=np.uint32)  # k = 0..7
    s = np.array([[1.0]], dtype=np.float16)
    b = np.array([[0.0]], dtype=np.float16)
    wq64 = np.tile(wq, (1, 8))  # 64 codes
    d = oracle.dequantize(wq64, s, b, group_size=64, bits=8)
    assert d[0, :8].tolist() == [1, 2, 3, 4, 127, 128, 0, 255]


# -------------------------------------------------------------------------
@pytest.mark.parametrize("N,K", [(8, 64), (33, 256), (100, 640), (17, 1024)])
def test_c_and_numpy_restatements_agree(N, K):
    w = synth.weight_fp16(N, K, seed=11)
    wq, s, b = oracle.quantize(w)
    wq2, s2, b2 = np_ref.quantize(w)
    np.testing.assert_array_equal(wq, wq2)
    np.testing.assert_array_equal(s.view(np.uint16), s2.view(np.uint16))
    np.testing.assert_array_equal(b.view(np.uint16), b2.view(np.uint16))
    for r, name in ((oracle.ROUND_TWICE, "twice"), (oracle.ROUND_ONCE, "once")):
        np.testing.assert_array_equal(oracle.dequantize(wq, s, b, rounding=r).view(np.uint16),
                                      np_ref.dequantize(wq, s, b, rounding=name).view(np.uint16))
    x = synth.activations(5, K, seed=11)
    y, y32 = oracle.quantized_matmul(x, wq, s, b, want_f32=True)
    y64 = np_ref.quantized_matmul(x, wq, s, b)
    assert rel_err(y32, y64) < 1e-5
    assert rel_err(y, y64) < 1e-3


def _sequential_f32(x, wq, s, b, gs, bits):
    """y32 by the oracle's stated arithmetic, one rounded float32 operation
    at a time: w = s*q, then w + b; then acc = acc + x*w over k ascending."""
    N = wq.shape[0]
    per = 32 // bits
    q = ((wq[:, :, None] >> (bits * np.arange(per, dtype=np.uint32))) & ((1 << bits) - 1)).reshape(N, -1)
    K = q.shape[1]
    s32 = np.repeat(s.astype(np.float32), gs, axis=1)
    b32 = np.repeat(b.astype(np.float32), gs, axis=1)
    w32 = (s32 * q.astype(np.float32)) + b32
    x32 = x.astype(np.float32)
    acc = np.zeros((x.shape[0], N), np.float32)
    for k in range(K):
        acc = acc + x32[:, k:k + 1] * w32[None, :, k]
    return acc


@pytest.mark.parametrize("bits,gs", [(4, 64), (4, 128), (8, 64), (8, 128)])
@pytest.mark.parametrize("M", [1, 3, 4, 5, 9])
def test_matmul_is_the_stated_float32_sequence(bits, gs, M):
    """Every path of the oracle's matmul -- the vectorised 16-row blocks
    (weights formed on the fly up to 4 rows of x, or from a dequantized block
    above), the scalar last block -- gives, bit for bit, the float32 sequence
    it is defined as."""
    N, K = 37, 512  # two full 16-row blocks and a partial one
    wq, s, b = oracle.quantize(synth.weight_fp16(N, K, seed=bits + gs + M), group_size=gs, bits=bits)
    x = synth.activations(M, K, seed=M)
    y, y32 = oracle.quantized_matmul(x, wq, s, b, group_size=gs, bits=bits, want_f32=True)
    ref = _sequential_f32(x, wq, s, b, gs, bits)
    np.testing.assert_array_equal(y32.view(np.uint32), ref.view(np.uint32))
    np.testing.assert_array_equal(y.view(np.uint16), ref.astype(np.float16).view(np.uint16))


def test_quantizer_reconstruction_error_is_bounded():
    w = synth.weight_fp16(64, 512, seed=5)
    wq, s, b = oracle.quantize(w)
    d = oracle.dequantize(wq, s, b).astype(np.float32)
    err = np.abs(d - w.astype(np.float32))
    smax = np.repeat(s.astype(np.float32), 64, axis=1)
    assert np.all(err <= 0.5 * smax + 2e-3)


# ---------------------------------------------------------------- fixtures
@pytest.mark.parametrize("name", golden_cases())
def test_golden_fixture_reproduces(name):
    g = load_golden(name)
    M, K = g["x"].shape
    N = g["wq"].shape[0]
    wq, s, b = g["wq"], g["scales"], g["biases"]
    np.testing.assert_array_equal(oracle.dequantize(wq, s, b).view(np.uint16), g["deq_twice"].view(np.uint16))
    np.testing.assert_array_equal(oracle.dequantize(wq, s, b, rounding=1).view(np.uint16),
                                  g["deq_once"].view(np.uint16))
    y, y32 = oracle.quantized_matmul(g["x"], wq, s, b, want_f32=True)
    np.testing.assert_array_equal(y.view(np.uint16), g["y"].view(np.uint16))
    np.testing.assert_array_equal(y32, g["y32"])
    assert rel_err(y32, np_ref.quantized_matmul(g["x"], wq, s, b)) < 1e-5
    assert y.shape == (M, N) and K == wq.shape[1] * 8


def test_golden_quantizer_inputs_regenerate():
    from tests.golden.gen_golden import CASES
    for name, (M, N, K, seed) in CASES.items():
        g = load_golden(name)
        w = synth.weight_fp16(N, K, seed=seed, layer=0, tid=0)
        wq, s, b = oracle.quantize(w)
        np.testing.assert_array_equal(wq, g["wq"])
        np.testing.assert_array_equal(s.view(np.uint16), g["scales"].view(np.uint16))
        np.testing.assert_array_equal(synth.activations(M, K, seed=seed), g["x"])


def test_full_size_configs_match_their_digests():
    """BASELINE's single configuration (17408 x 5120 at M = 1 and 16) and an
    8-bit, group-128 override shape at full size: the oracle's quantized
    triple and outputs, regenerated from the seeds, hash to the committed
    digests (tests/golden/baseline_digests.json)."""
    import json
    from tests.golden.gen_golden import DIGEST_FILE, digest_cases
    with open(DIGEST_FILE) as f:
        committed = json.load(f)
    assert digest_cases() == committed


def test_swiglu_known_answer():
    """The reference's activation test input (ffi_tests.rs:1536-1548: gate
    [1, 2, 3, 4], x = 2 everywhere, positive sum) against silu(g) * x in
    float64, within the fp16 rounding of the three ops."""
    gate = np.array([[1.0, 2.0, 3.0, 4.0]], np.float16)
    x = np.full((1, 4), 2.0, np.float16)
    out = oracle.swiglu(gate, x)
    g = gate.astype(np.float64)
    exact = g / (1.0 + np.exp(-g)) * 2.0
    assert out.dtype == np.float16 and out.shape == (1, 4)
    assert float(out.astype(np.float64).sum()) > 0.0
    np.testing.assert_allclose(out.astype(np.float64), exact, rtol=2e-3)


def test_swiglu_special_values():
    """Large negative gates give zero (sigmoid underflows), large positive
    ones pass gate * up through; zeros stay zero."""
    gate = np.array([-65504.0, -100.0, -20.0, 0.0, 20.0, 100.0], np.float16)
    up = np.array([1.0, 1.0, 1.0, 5.0, 1.0, 1.0], np.float16)
    out = oracle.swiglu(gate, up).astype(np.float64)
    assert out[0] == 0.0 and out[1] == 0.0 and out[3] == 0.0
    assert abs(out[2]) < 1e-6
    assert out[4] == 20.0 and out[5] == 100.0


def test_swiglu_matmul_is_op_by_op():
    """quantized_matmul_swiglu is the two fp16 matmuls followed by the
    activation (compiled and uncompiled forms agree, ffi_tests.rs:3020-3060)."""
    gate = oracle.quantize(synth.weight_fp16(72, 256, seed=1))
    up = oracle.quantize(synth.weight_fp16(72, 256, seed=2))
    x = synth.activations(3, 256, seed=3)
    h = oracle.quantized_matmul_swiglu(x, gate, up)
    g = oracle.quantized_matmul(x, *gate).astype(np.float32)
    u = oracle.quantized_matmul(x, *up).astype(np.float32)
    sig = (1.0 / (1.0 + np.exp(-g))).astype(np.float16).astype(np.float32)
    ref = ((g * sig).astype(np.float16).astype(np.float32) * u).astype(np.float16)
    np.testing.assert_array_equal(h.view(np.uint16), ref.view(np.uint16))


def test_topk_reference_candidate_vectors():
    """The reference's candidate test vectors (qwen3_5_dflash.rs:3884-3928):
    four peaks over a flat floor, in the compact domain (80,922 logits at
    -1000) and the full vocabulary (248,320 at -2000), give exactly the peaks.
    The id remapping between the two domains is the DFlash drafter's, outside
    this path, so each domain is checked on its own ids."""
    peaks = {0: 40.0, 80_000: 50.0, 80_001: 60.0, 80_921: 70.0}
    for n, floor in ((80_922, -1000.0), (248_320, -2000.0)):
        logits = np.full((1, 1, n), floor, np.float16)
        for i, v in peaks.items():
            logits[0, 0, i] = v
        idx, vals = oracle.topk(logits, len(peaks))
        assert idx.shape == (1, 1, 4)
        assert dict(zip(idx[0, 0].tolist(), vals[0, 0].astype(float).tolist())) == peaks
        assert idx[0, 0].tolist() == [80_921, 80_001, 80_000, 0]  # descending by value


def test_topk_bounds_and_ties():
    """k must lie in 1..N-1 (qwen3_5_dflash.rs:3931-3938); equal values keep
    the lower indices, and -0 sorts below +0."""
    z = np.zeros((1, 1, 4), np.float16)
    for bad in (0, 4, 5):
        with pytest.raises(ValueError):
            oracle.topk(z, bad)
    idx, _ = oracle.topk(z, 1)
    assert idx.tolist() == [[[0]]]
    row = np.array([[1, 3, 3, 2, 3, 3, -0.0, 0.0]], np.float16)
    idx, vals = oracle.topk(row, 3)
    assert idx.tolist() == [[1, 2, 4]] and vals.astype(float).tolist() == [[3, 3, 3]]
    idx, _ = oracle.topk(row, 7)
    assert idx.tolist() == [[1, 2, 4, 5, 3, 0, 7]]
