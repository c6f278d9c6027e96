"""The decode kernel's schedule choices (qw_decode_schedule, computed on the
host; no GPU needed) for the BASELINE 27B stack's shapes on a 148-SM B200:
16-group units where they do not leave the busiest CTA with more than 10%
more k (and keep TMA scales), clusters of 2 or 3 CTAs per row tile for the
few-tile shapes, whole tiles per CTA for the fused SwiGLU launch, stream-K
for the LM head."""
import pytest

import qw_b200
from qw_b200 import synth, tp

SM = 148


def sched(M, N, K, **kw):
    return qw_b200.decode_schedule(M, N, K, sm_count=SM, **kw)


def test_one_token_stack_shapes():
    # q|k|v: 16-group units would give 3 units of 1024 k against 5 of 512
    assert sched(1, 8192, 5120) == {"tokens": 1, "unit_k": 512, "ctas": 128, "split": 2, "busiest_units": 5}
    assert sched(1, 5120, 6144) == {"tokens": 1, "unit_k": 1024, "ctas": 120, "split": 3, "busiest_units": 2}
    assert sched(1, 5120, 17408) == {"tokens": 1, "unit_k": 1024, "ctas": 120, "split": 3, "busiest_units": 6}
    # fused SwiGLU gate|up: 272 tiles of 64 outputs, two whole tiles on each of 136 CTAs
    assert sched(1, 17408, 5120, swiglu=True) == {"tokens": 1, "unit_k": 1024, "ctas": 136, "split": 1,
                                                   "busiest_units": 10}
    # LM head: stream-K over every SM
    assert sched(1, 151936, 5120) == {"tokens": 1, "unit_k": 1024, "ctas": 148, "split": 1, "busiest_units": 41}
    # BASELINE single configuration: one 17408-row matmul, 136 tiles, one CTA each
    assert sched(1, 17408, 5120) == {"tokens": 1, "unit_k": 1024, "ctas": 136, "split": 1, "busiest_units": 5}


def test_one_token_keeps_tma_scales():
    """K a multiple of 512 but not of 1024 (the down shard at TP=2): 8-group
    units keep the TMA path for scales and biases."""
    N, K = tp.shard_shape(synth.layer_linears()[3], 2)
    assert (N, K) == (5120, 8704)
    assert sched(1, N, K)["unit_k"] == 512


@pytest.mark.parametrize("M,tokens", [(2, 4), (4, 4), (5, 8), (8, 8), (9, 16), (16, 16)])
def test_configuration_by_rows(M, tokens):
    s = sched(M, 17408, 5120)
    assert s["tokens"] == tokens and s["unit_k"] == 512


@pytest.mark.parametrize("M", [4, 16])
def test_swiglu_whole_tiles_within_ten_percent(M):
    """20 units a CTA in whole tiles against 19 under stream-K: whole tiles."""
    assert sched(M, 17408, 5120, swiglu=True) == {"tokens": M, "unit_k": 512, "ctas": 136, "split": 1,
                                                   "busiest_units": 20}


def test_eight_bit_codes():
    assert sched(1, 17408, 5120, bits=8)["tokens"] == 1
    assert sched(1, 17408, 5120, bits=8)["unit_k"] == 512


def test_rejects_outside_the_decode_kernel():
    from qw_b200._lib import QwError
    with pytest.raises(QwError):
        sched(17, 17408, 5120)   # 17 rows take the tensor-core kernel
    with pytest.raises(QwError):
        sched(1, 17408, 5100)    # K not a multiple of the group
    with pytest.raises(QwError):
        sched(1, 17408, 5120, bits=3)
