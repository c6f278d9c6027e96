"""qw_quantized_matmul_static_scratch through the C ABI, against
qw_quantized_matmul on the same inputs.

The entry point keeps its scratch in one fixed device array shared by every
call, so each case makes two calls in a row with different activations before
either result is read: the second call runs on whatever the first left in
the array.  Shapes cover the three schedules of the skinny kernel: one CTA per
row tile, a cluster splitting each tile (partials reduced in shared memory),
and stream-K over more tiles than SMs (split-tile counters and partial sums in
the scratch).  A fresh process also checks the property the entry point
exists for: once its kernels are loaded, repeated calls, on the first stream
and on new ones, and a read of the status words leave the device's free
memory unchanged, while the allocating entry point on a new stream lowers it.  This file is collected last so that it also runs after every
other test in the same process; it passes alone in a fresh process as well.
Tolerance: max |y - y_ref| <= 1e-2 * rms(y_ref)."""
import ctypes
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from qw_b200 import _lib
from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu

_DT = {torch.float16: _lib.QW_F16, torch.float32: _lib.QW_F32, torch.int32: _lib.QW_U32}


def _arr(t):
    a = _lib.QwArray()
    a.data = t.data_ptr()
    a.dtype = _DT[t.dtype]
    a.ndim = t.dim()
    for i, (s, st) in enumerate(zip(t.shape, t.stride())):
        a.shape[i] = s
        a.strides[i] = st
    return ctypes.pointer(a)


def _call(fn_name, x, wq, s, b, y):
    fn = getattr(_lib.load(), fn_name)
    stream = torch.cuda.current_stream().cuda_stream
    return fn(_arr(x), _arr(wq), _arr(s), _arr(b), 1, 64, 4, b"affine", _arr(y), stream)


def _weights(N, K, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.02).half()
    import qw_b200
    return qw_b200.quantize_weights(w)


def _x(M, K, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(M, K, generator=g, device="cuda").half()


@pytest.mark.parametrize("M,N,K,out_dtype", [
    (1, 17408, 5120, torch.float16),    # 136 row tiles: one CTA per tile
    (4, 5120, 17408, torch.float16),    # 40 row tiles: clusters split each tile
    (16, 40064, 5120, torch.float16),   # 313 row tiles: stream-K, counters + partials
    (1, 151936, 5120, torch.float32),   # lm_head width, fp32 accumulators out
])
def test_two_calls_in_a_row_match_qw_quantized_matmul(cuda_dev, M, N, K, out_dtype):
    wq, s, b = _weights(N, K, seed=N + M)
    x1, x2 = _x(M, K, seed=1), _x(M, K, seed=2)
    y1 = torch.full((M, N), float("nan"), device="cuda", dtype=out_dtype)
    y2 = torch.full((M, N), float("nan"), device="cuda", dtype=out_dtype)
    _lib.check(_call("qw_quantized_matmul_static_scratch", x1, wq, s, b, y1))
    _lib.check(_call("qw_quantized_matmul_static_scratch", x2, wq, s, b, y2))
    r1 = torch.empty((M, N), device="cuda", dtype=out_dtype)
    r2 = torch.empty((M, N), device="cuda", dtype=out_dtype)
    _lib.check(_call("qw_quantized_matmul", x1, wq, s, b, r1))
    _lib.check(_call("qw_quantized_matmul", x2, wq, s, b, r2))
    torch.cuda.synchronize()
    for y, r in ((y1, r1), (y2, r2)):
        y_np, r_np = y.float().cpu().numpy(), r.float().cpu().numpy()
        assert np.isfinite(y_np).all()
        assert rel_err(y_np, r_np) <= TOL


def test_rejects_more_than_16_rows(cuda_dev):
    N, K = 256, 512
    wq, s, b = _weights(N, K, seed=3)
    x = _x(17, K, seed=3)
    y = torch.zeros((17, N), device="cuda", dtype=torch.float16)
    rc = _call("qw_quantized_matmul_static_scratch", x, wq, s, b, y)
    assert rc == _lib.QW_EUNSUPPORTED
    assert "at most 16 rows" in _lib.load().qw_last_error().decode()
    torch.cuda.synchronize()
    assert not y.any()


_FRESH_PROCESS = r"""
import ctypes, json, sys
import torch
sys.path.insert(0, sys.argv[1])
from tests.test_zz_no_alloc import _arr, _weights, _x
from qw_b200 import _lib
L = _lib.load()
shapes = [(1, 17408, 5120), (4, 5120, 17408), (16, 40064, 5120)]
cases = []
for M, N, K in shapes:
    wq, s, b = _weights(N, K, seed=N)
    cases.append((_x(M, K, seed=M), wq, s, b, torch.empty(M, N, device="cuda", dtype=torch.float16)))
streams = [torch.cuda.Stream() for _ in range(3)]
torch.cuda.synchronize()

def static_calls(stream):
    for x, wq, s, b, y in cases:
        _lib.check(L.qw_quantized_matmul_static_scratch(_arr(x), _arr(wq), _arr(s), _arr(b), 1, 64, 4,
                                                        b"affine", _arr(y), stream))

static_calls(torch.cuda.current_stream().cuda_stream)  # loads the kernels and resolves the array
torch.cuda.synchronize()
free0 = torch.cuda.mem_get_info()[0]
for _ in range(3):
    static_calls(torch.cuda.current_stream().cuda_stream)
for st in streams:
    static_calls(st.cuda_stream)
torch.cuda.synchronize()
st_word = ctypes.c_uint(7)
_lib.check(L.qw_device_status(torch.cuda.current_device(), ctypes.byref(st_word), 1))
free1 = torch.cuda.mem_get_info()[0]
# control: the allocating entry point's scratch for a stream-K shape on a new stream
x, wq, s, b, y = cases[2]
fresh = torch.cuda.Stream()
_lib.check(L.qw_quantized_matmul(_arr(x), _arr(wq), _arr(s), _arr(b), 1, 64, 4, b"affine", _arr(y),
                                 fresh.cuda_stream))
torch.cuda.synchronize()
free2 = torch.cuda.mem_get_info()[0]
print(json.dumps({"free0": free0, "free1": free1, "free2": free2, "status": st_word.value}))
"""


def test_allocates_nothing_in_a_fresh_process(cuda_dev):
    """Free device memory (cudaMemGetInfo) is the same before and after
    repeated static-scratch calls on the first stream and on three new
    streams, plus a qw_device_status read: no per-stream scratch and no
    status word were allocated.  The same shape through qw_quantized_matmul
    on a new stream allocates its scratch and lowers free memory, which shows
    the measurement sees an allocation of that size."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-c", _FRESH_PROCESS, root], capture_output=True, text=True,
                         timeout=600, cwd=root)
    assert out.returncode == 0, out.stderr[-2000:]
    r = json.loads(out.stdout.strip().splitlines()[-1])
    assert r["status"] == 0
    assert r["free1"] == r["free0"], r
    assert r["free2"] < r["free1"], r
