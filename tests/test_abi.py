"""CPU tests of the C ABI: the library loads, exports every entry point its
header declares, and rejects invalid arguments with the reference's
validation rules before touching a device.  No GPU."""
import ctypes
import os
import re
import subprocess

import pytest

from qw_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include")))
           if f.endswith(".h")]


def declared_functions():
    names = []
    for h in HEADERS:
        text = open(h).read()
        names += re.findall(r"^\s*(?:int|const char\s*\*|size_t|void)\s+(qw\w+)\s*\(", text, re.M)
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("qw_quantized_matmul", "qw_quantized_linear_forward", "qw_dequantize", "qw_quantize",
                     "qw_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    for name in declared_functions():
        assert hasattr(L, name), f"{name} declared in include/ but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (qw_\w+)", out))
    assert set(declared_functions()) <= exported


def test_python_signatures_cover_the_header():
    # every entry point the header declares has a ctypes signature in _lib
    assert set(declared_functions()) <= set(_lib.SIGNATURES)


def test_abi_version():
    assert _lib.load().qw_abi_version() == 1


def _arr(shape, dtype, ptr=0x1000):
    a = _lib.QwArray()
    a.data = ptr
    a.dtype = dtype
    a.ndim = len(shape)
    for i, s in enumerate(shape):
        a.shape[i] = s
    return ctypes.pointer(a)


def _qmm(x, w, s, b, mode=b"affine", gs=64, bits=4, y=None, transpose=1):
    L = _lib.load()
    return L.qw_quantized_matmul(x, w, s, b, transpose, gs, bits, mode, y, None)


def std_args(M=1, N=256, K=512):
    return (_arr([M, K], _lib.QW_F16), _arr([N, K // 8], _lib.QW_U32), _arr([N, K // 64], _lib.QW_F16),
            _arr([N, K // 64], _lib.QW_F16), _arr([M, N], _lib.QW_F16))


def err():
    return _lib.load().qw_last_error().decode()


def test_rejects_unknown_mode():
    x, w, s, b, y = std_args()
    assert _qmm(x, w, s, b, mode=b"Affine", y=y) == _lib.QW_EINVAL
    assert "mode" in err()


def test_block_float_modes_are_unsupported_not_invalid():
    x, w, s, b, y = std_args()
    assert _qmm(x, w, s, None, mode=b"mxfp4", y=y) == _lib.QW_EUNSUPPORTED


def test_affine_requires_biases():
    x, w, s, b, y = std_args()
    assert _qmm(x, w, s, None, y=y) == _lib.QW_EINVAL
    assert "biases" in err()


def test_biases_with_block_float_mode_rejected():
    x, w, s, b, y = std_args()
    assert _qmm(x, w, s, b, mode=b"nvfp4", y=y) == _lib.QW_EINVAL


@pytest.mark.parametrize("bits,gs,code", [(0, 64, _lib.QW_EINVAL), (33, 64, _lib.QW_EINVAL),
                                          (4, 0, _lib.QW_EINVAL), (4, (1 << 20) + 1, _lib.QW_EINVAL),
                                          (2, 64, _lib.QW_EUNSUPPORTED), (4, 32, _lib.QW_EUNSUPPORTED),
                                          (6, 64, _lib.QW_EUNSUPPORTED), (8, 256, _lib.QW_EUNSUPPORTED)])
def test_bits_and_group_bounds(bits, gs, code):
    """Bounds of layers.rs:1286-1318; in-range values other than bits 4/8 with
    groups of 64/128 are unsupported."""
    x, w, s, b, y = std_args()
    assert _qmm(x, w, s, b, gs=gs, bits=bits, y=y) == code


def test_packing_invariant():
    x, _, s, b, y = std_args()
    w_bad = _arr([256, 63], _lib.QW_U32)
    assert _qmm(x, w_bad, s, b, y=y) == _lib.QW_EINVAL
    assert "packed width" in err()


def test_biases_shape_must_match_scales():
    x, w, s, _, y = std_args()
    b_bad = _arr([256, 7], _lib.QW_F16)
    assert _qmm(x, w, s, b_bad, y=y) == _lib.QW_EINVAL


def test_x_width_must_match():
    _, w, s, b, y = std_args()
    x_bad = _arr([1, 448], _lib.QW_F16)
    assert _qmm(x_bad, w, s, b, y=y) == _lib.QW_EINVAL


def test_output_shape_checked():
    x, w, s, b, _ = std_args()
    assert _qmm(x, w, s, b, y=_arr([1, 255], _lib.QW_F16)) == _lib.QW_EINVAL


def _arr_strided(shape, strides, dtype, ptr=0x1000):
    a = _arr(shape, dtype, ptr)
    for i, st in enumerate(strides):
        a.contents.strides[i] = st
    return a


def test_row_strided_x_layouts():
    """x may be a column slice (rows of K, one row stride, 16-byte aligned);
    anything else is rejected before any device work."""
    _, w, s, b, y = std_args(M=4)
    # row stride 516: not a multiple of 8 elements (rows would lose 16-byte alignment)
    assert _qmm(_arr_strided([4, 512], [516, 1], _lib.QW_F16), w, s, b, y=y) == _lib.QW_EINVAL
    assert "multiple of 8" in err()
    # overlapping rows
    assert _qmm(_arr_strided([4, 512], [256, 1], _lib.QW_F16), w, s, b, y=y) == _lib.QW_EINVAL
    assert "overlap" in err()
    # last dimension not contiguous
    assert _qmm(_arr_strided([4, 512], [1024, 2], _lib.QW_F16), w, s, b, y=y) == _lib.QW_EINVAL
    assert "last dimension" in err()
    # leading dimensions that do not collapse into one row index
    y3 = _arr([2, 2, 256], _lib.QW_F16)
    assert _qmm(_arr_strided([2, 2, 512], [4096, 1024, 1], _lib.QW_F16), w, s, b, y=y3) == _lib.QW_EINVAL
    assert "leading dimensions" in err()


def test_transpose_false_unsupported():
    x, w, s, b, y = std_args()
    assert _qmm(x, w, s, b, y=y, transpose=0) == _lib.QW_EUNSUPPORTED


def test_unsupported_activation_dtype():
    _, w, s, b, y = std_args()
    assert _qmm(_arr([1, 512], _lib.QW_BF16), w, s, b, y=y) == _lib.QW_EUNSUPPORTED


def test_empty_problem_is_a_no_op():
    _, w, s, b, _ = std_args()
    x0 = _arr([0, 512], _lib.QW_F16, ptr=0)
    y0 = _arr([0, 256], _lib.QW_F16, ptr=0)
    assert _qmm(x0, w, s, b, y=y0) == _lib.QW_OK


def test_misaligned_weights_rejected():
    x, _, s, b, y = std_args()
    w_mis = _arr([256, 64], _lib.QW_U32, ptr=0x1004)
    assert _qmm(x, w_mis, s, b, y=y) == _lib.QW_EINVAL
    assert "aligned" in err()


# ---- the later entry points' argument checks (all before any device work)

def test_swiglu_requires_matching_gate_and_up():
    L = _lib.load()
    x, w, s, b, _ = std_args(N=256)
    w_up, s_up, b_up = _arr([128, 64], _lib.QW_U32), _arr([128, 8], _lib.QW_F16), _arr([128, 8], _lib.QW_F16)
    y = _arr([1, 256], _lib.QW_F16)
    assert L.qw_quantized_matmul_swiglu(x, w, s, b, w_up, s_up, b_up, 1, 64, 4, b"affine", y, None) == \
        _lib.QW_EINVAL
    assert "same shape" in err()
    assert L.qw_quantized_matmul_swiglu(x, w, s, b, w, s, None, 1, 64, 4, b"affine", y, None) == _lib.QW_EINVAL
    assert "requires biases" in err()
    assert L.qw_quantized_matmul_swiglu(x, w, s, b, w, s, b, 1, 64, 2, b"affine", y, None) in \
        (_lib.QW_EINVAL, _lib.QW_EUNSUPPORTED)


def test_swiglu_activation_shapes():
    L = _lib.load()
    g, u = _arr([2, 8], _lib.QW_F16), _arr([2, 8], _lib.QW_F16)
    assert L.qw_swiglu_activation(g, _arr([8, 2], _lib.QW_F16), _arr([2, 8], _lib.QW_F16), None) == _lib.QW_EINVAL
    assert L.qw_swiglu_activation(g, u, _arr([2, 8], _lib.QW_F32), None) == _lib.QW_EUNSUPPORTED


@pytest.mark.parametrize("k,code", [(0, _lib.QW_EINVAL), (4096, _lib.QW_EINVAL), (5000, _lib.QW_EINVAL),
                                    (1025, _lib.QW_EUNSUPPORTED)])
def test_topk_bounds(k, code):
    L = _lib.load()
    logits = _arr([2, 4096], _lib.QW_F16)
    idx = _arr([2, max(k, 1)], _lib.QW_U32)
    assert L.qw_topk(logits, k, idx, None, None) == code


def test_topk_output_shapes():
    L = _lib.load()
    logits = _arr([2, 4096], _lib.QW_F16)
    assert L.qw_topk(logits, 16, _arr([2, 8], _lib.QW_U32), None, None) == _lib.QW_EINVAL
    assert L.qw_topk(logits, 16, _arr([2, 16], _lib.QW_F16), None, None) == _lib.QW_EINVAL
    assert L.qw_topk(logits, 16, _arr([2, 16], _lib.QW_U32), _arr([2, 16], _lib.QW_F32), None) == _lib.QW_EINVAL
    assert L.qw_topk(_arr([2, 4096], _lib.QW_F32), 16, _arr([2, 16], _lib.QW_U32), None, None) == \
        _lib.QW_EUNSUPPORTED


def test_allreduce_init_bounds():
    L = _lib.load()
    comm = ctypes.c_void_p()
    h = ctypes.create_string_buffer(_lib.QW_IPC_HANDLE_BYTES)
    assert L.qw_allreduce_init(9, 0, 1024, ctypes.byref(comm), h) == _lib.QW_EUNSUPPORTED
    assert L.qw_allreduce_init(2, 2, 1024, ctypes.byref(comm), h) == _lib.QW_EINVAL
    assert L.qw_allreduce_init(2, 0, 0, ctypes.byref(comm), h) == _lib.QW_EINVAL
    assert L.qw_allreduce_sum(None, _arr([4], _lib.QW_F32), _arr([4], _lib.QW_F16), None) == _lib.QW_EINVAL
    assert L.qw_allreduce_matmul(None, _arr([1, 64], _lib.QW_F16), _arr([8, 8], _lib.QW_U32),
                                 _arr([8, 1], _lib.QW_F16), _arr([8, 1], _lib.QW_F16), 64, 4, b"affine",
                                 _arr([1, 8], _lib.QW_F16), None) == _lib.QW_EINVAL
    assert b"comm is null" in L.qw_last_error()
    assert L.qw_allreduce_destroy(None) == _lib.QW_OK
