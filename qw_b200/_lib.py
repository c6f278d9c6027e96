"""ctypes binding of libqwqmm.so (include/qw_qmm.h).

The library is built in-tree (``make -C qw_b200/csrc``) and loaded from this
directory.  There is no fallback: if the library is missing the import of the
operators fails loudly.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqwqmm.so")

QW_OK = 0
QW_EINVAL = 1
QW_EUNSUPPORTED = 2
QW_ECUDA = 3
QW_ETIMEOUT = 4
QW_ENOMEM = 5

QW_U32 = 1
QW_F16 = 2
QW_BF16 = 3
QW_F32 = 4

QW_IPC_HANDLE_BYTES = 64

# Every entry point include/qw_qmm.h declares, with its ctypes signature.
_P = ctypes.c_void_p
_I = ctypes.c_int


class QwArray(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dtype", ctypes.c_int32),
        ("ndim", ctypes.c_int32),
        ("shape", ctypes.c_int64 * 4),
        ("strides", ctypes.c_int64 * 4),
    ]


_PA = ctypes.POINTER(QwArray)


class QwQmmOp(ctypes.Structure):
    _fields_ = [("x", _PA), ("w", _PA), ("scales", _PA), ("biases", _PA), ("y", _PA)]


SIGNATURES = {
    "qw_quantized_matmul": ([_PA, _PA, _PA, _PA, _I, _I, _I, ctypes.c_char_p, _PA, _P], _I),
    "qw_quantized_matmul_argmax": ([_PA, _PA, _PA, _PA, _I, _I, ctypes.c_char_p, _PA, _PA, _P], _I),
    "qw_quantized_matmul_chain": ([ctypes.POINTER(QwQmmOp), _I, _I, _I, ctypes.c_char_p, _P], _I),
    "qw_topk": ([_PA, _I, _PA, _PA, _P], _I),
    "qw_allreduce_init": ([_I, _I, ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p], _I),
    "qw_allreduce_connect": ([ctypes.c_void_p, ctypes.c_char_p], _I),
    "qw_allreduce_sum": ([ctypes.c_void_p, _PA, _PA, _P], _I),
    "qw_allreduce_destroy": ([ctypes.c_void_p], _I),
    "qw_decode_schedule": ([ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _I, _I, _I, _I,
                            ctypes.POINTER(ctypes.c_int64)], _I),
    "qw_allreduce_matmul": ([ctypes.c_void_p, _PA, _PA, _PA, _PA, _I, _I, ctypes.c_char_p, _PA, _P], _I),
    "qw_allreduce_argmax": ([ctypes.c_void_p, _PA, _PA, _PA, _PA, _I, _I, ctypes.c_char_p, ctypes.c_int64, _PA, _PA,
                             _P], _I),
    "qw_quantized_matmul_topk": ([_PA, _PA, _PA, _PA, _I, _I, ctypes.c_char_p, _I, _PA, _PA, _PA, _P], _I),
    "qw_quantized_matmul_swiglu": ([_PA, _PA, _PA, _PA, _PA, _PA, _PA, _I, _I, _I, ctypes.c_char_p, _PA, _P], _I),
    "qw_swiglu_activation": ([_PA, _PA, _PA, _P], _I),
    "qw_swiglu_mlp": ([_PA, _PA, _PA, _PA, _PA, _PA, _PA, _PA, _PA, _PA, _I, _I, ctypes.c_char_p, _PA, _P], _I),
    "qw_quantized_matmul_static_scratch": ([_PA, _PA, _PA, _PA, _I, _I, _I, ctypes.c_char_p, _PA, _P], _I),
    "qw_quantized_linear_forward": ([_PA, _PA, _PA, _PA, _PA, _I, _I, ctypes.c_char_p, _PA, _P], _I),
    "qw_quantized_linear_forward_global_scale": (
        [_PA, _PA, _PA, _PA, _PA, _PA, _I, _I, ctypes.c_char_p, _PA, _P], _I),
    "qw_dequantize": ([_PA, _PA, _PA, _I, _I, ctypes.c_char_p, _PA, _P], _I),
    "qw_dequantize_rounding": ([_PA, _PA, _PA, _I, _I, ctypes.c_char_p, _I, _PA, _P], _I),
    "qw_quantize": ([_PA, _I, _I, ctypes.c_char_p, _PA, _PA, _PA, _P], _I),
    "qw_last_error": ([], ctypes.c_char_p),
    "qw_device_status": ([_I, ctypes.POINTER(ctypes.c_uint), _I], _I),
    "qw_abi_version": ([], _I),
}

_lib = None


class QwError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"qw status {code}: {msg}")
        self.code = code


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `make -C qw_b200/csrc` "
                "(there is no CPU fallback for the quantized matmul)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(rc: int):
    if rc != QW_OK:
        raise QwError(rc, load().qw_last_error().decode())
