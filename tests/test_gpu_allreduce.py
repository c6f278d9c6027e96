"""The one-shot peer allreduce (qw_allreduce_sum) on P GPUs, one process per
GPU: every rank gets the fp32 partials summed in rank order, bit for bit the
float32 sum numpy forms in the same order (and its fp16 rounding); sizes that
are and are not multiples of the 4-float vector; repeated calls, eager and
replayed from a CUDA graph (the epoch advances on the device); calls of
different sizes (so different grids and chunk boundaries) issued back to back
with no host synchronization while one rank starts each call late; and a
rank whose peer never calls gives up after the bounded wait with a timeout
status instead of hanging.

The row-parallel matmul with the exchange fused into the decode kernel's
epilogue (qw_allreduce_matmul) equals, bit for bit and on every rank, the
same rank's qw_quantized_matmul into fp32 followed by qw_allreduce_sum:
cluster-split and stream-K schedules (split tiles finished by whichever CTA
arrives last), ragged N, 1 to 16 rows, 8-bit codes, the M > 16 path that
runs the two kernels, graph replay, fused calls interleaved with plain sums
with no host synchronization and a late rank, and the bounded wait when a
peer never calls.  Needs at least 2 GPUs (skipped otherwise); NVLS off."""
import os
import socket
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

SIZES = [5120, 5121, 16 * 5120, 3]
# Back-to-back calls whose grids differ: 148 chunks (a prefill-sized vector),
# 3 (one decode row), 40 (sixteen rows), 1, ...
MIXED = [64 * 5120, 5120, 64 * 5120, 16 * 5120, 3, 5121, 64 * 5120, 16 * 5120, 5120] * 3
# Row-parallel matmuls (M, N, K per rank, bits): the o and down shards of the
# 27B layer at TP 8 and 2 (clusters of 2 and 3 CTAs per 128-row tile), 313
# tiles over 148 CTAs (stream-K, split tiles), 296 tiles two to a CTA (whole
# tiles), 136 tiles (one CTA each), ragged N and M, 8-bit codes, and M = 17
# (the matmul and the allreduce kernel).
MATMULS = [(1, 5120, 768, 4), (1, 5120, 2176, 4), (4, 5120, 3072, 4), (16, 5120, 8704, 4), (1, 40000, 2048, 4),
           (1, 37888, 1024, 4), (3, 1000, 512, 4), (8, 17408, 1024, 4), (2, 5120, 1024, 8), (17, 5120, 1024, 4)]
MM_MAX = max(m * n for m, n, _, _ in MATMULS)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partial(rank, n, step):
    rng = np.random.default_rng(1000 * step + 17 * rank + n)
    return rng.standard_normal(n).astype(np.float32) * 4


def _expected(world, n, step):
    s = np.zeros(n, np.float32)
    for r in range(world):
        s = s + _partial(r, n, step)  # rank order, float32
    return s


def _matmul_case(rank, i, M, N, K, bits, dev):
    """This rank's K-slice of case i: x [M, K] and quantized w [N, K]."""
    from qw_b200 import ops
    g = torch.Generator(device="cpu").manual_seed(7919 * i + 101 * rank + 1)
    x = (torch.randn(M, K, generator=g) * 0.5).half().to(dev)
    w = (torch.randn(N, K, generator=g) * K ** -0.5).half().to(dev)
    return x, ops.quantize_weights(w, bits=bits)


def _unfused(ar, x, w, bits, dtype):
    """The two-kernel statement: this rank's fp32 product, then the sum."""
    from qw_b200 import ops
    part = ops.quantized_matmul(x, *w, bits=bits, out_dtype=torch.float32)
    return ar(part, torch.empty(part.shape, dtype=dtype, device=part.device))


def _rank_main(rank, world, port, out_q, scenario):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    from qw_b200 import ops, tp
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        ar = tp.PeerAllreduce(max(SIZES + MIXED + [MM_MAX]))
        if scenario == "matmul":
            results = []
            for i, (M, N, K, bits) in enumerate(MATMULS):
                x, w = _matmul_case(rank, i, M, N, K, bits, dev)
                for dtype in (torch.float16, torch.float32):
                    y = ar.matmul(x, w, torch.empty(M, N, dtype=dtype, device=dev), bits=bits)
                    ref = _unfused(ar, x, w, bits, dtype)
                    torch.cuda.synchronize()
                    results.append((i, str(dtype), y.cpu().numpy(), ref.cpu().numpy()))
            # graph: two fused calls and a plain sum captured, replayed with new x
            x1, w1 = _matmul_case(rank, 50, 1, 5120, 768, 4, dev)
            x2, w2 = _matmul_case(rank, 51, 4, 5120, 2176, 4, dev)
            part = torch.zeros(5120, dtype=torch.float32, device=dev)
            ys = [torch.empty(1, 5120, dtype=torch.float16, device=dev), torch.empty(5120, dtype=torch.float16, device=dev),
                  torch.empty(4, 5120, dtype=torch.float16, device=dev)]
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):  # the stream's scratch exists before capture
                ar.matmul(x1, w1, ys[0])
                ar(part, ys[1])
                ar.matmul(x2, w2, ys[2])
            s.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                ar.matmul(x1, w1, ys[0])
                ar(part, ys[1])
                ar.matmul(x2, w2, ys[2])
            graph_results = []
            for step in range(3):
                x1.copy_(_matmul_case(rank, 60 + step, 1, 5120, 768, 4, dev)[0])
                x2.copy_(_matmul_case(rank, 70 + step, 4, 5120, 2176, 4, dev)[0])
                part.copy_(torch.from_numpy(_partial(rank, 5120, 200 + step)))
                torch.cuda.synchronize()
                with torch.cuda.stream(s):
                    g.replay()
                s.synchronize()
                refs = [_unfused(ar, x1, w1, 4, torch.float16), _unfused(ar, x2, w2, 4, torch.float16)]
                torch.cuda.synchronize()
                graph_results.append(([y.cpu().numpy() for y in ys], [t.cpu().numpy() for t in refs]))
            del g
            dist.barrier()
            out_q.put((rank, "ok", (results, graph_results, ops.device_status(rank, clear=True))))
        elif scenario == "matmul_mixed":
            # references first (synchronized), then fused matmuls and plain
            # sums queued back to back with no host sync, the last rank late
            cases = [_matmul_case(rank, i, M, N, K, bits, dev) for i, (M, N, K, bits) in enumerate(MATMULS)]
            refs = [_unfused(ar, x, w, MATMULS[i][3], torch.float16) for i, (x, w) in enumerate(cases)]
            parts = [torch.from_numpy(_partial(rank, n, 700 + i)).to(dev) for i, n in enumerate(MIXED[:len(cases)])]
            torch.cuda.synchronize()
            dist.barrier()
            outs = []
            for rep in range(2):
                for i, ((x, w), part) in enumerate(zip(cases, parts)):
                    if rank == world - 1:
                        torch.cuda._sleep(20000 + 15000 * (i % 4))
                    M, N, _, bits = MATMULS[i]
                    outs.append(ar.matmul(x, w, torch.empty(M, N, dtype=torch.float16, device=dev), bits=bits))
                    outs.append(ar(part, torch.empty(part.shape, dtype=torch.float16, device=dev)))
            torch.cuda.synchronize()
            out_q.put((rank, "ok", ([t.cpu().numpy() for t in refs], [t.cpu().numpy() for t in outs],
                                    ops.device_status(rank, clear=True))))
            dist.barrier()
        elif scenario == "matmul_timeout":  # rank 1 never calls
            st = 0
            t = 0.0
            if rank == 0:
                x, w = _matmul_case(rank, 0, 1, 5120, 768, 4, dev)
                y = torch.empty(1, 5120, dtype=torch.float16, device=dev)
                torch.cuda.synchronize()
                ops.device_status(rank, clear=True)
                t0 = time.time()
                ar.matmul(x, w, y)
                torch.cuda.synchronize()
                t = time.time() - t0
                st = ops.device_status(rank, clear=True)
            dist.barrier()
            out_q.put((rank, "ok", (st, t)))
        elif scenario == "mixed":
            # every partial uploaded first, then all calls queued on one
            # stream without a host sync; the last rank starts each call late
            # (a bounded device spin before it), so the others run ahead
            parts = [torch.from_numpy(_partial(rank, n, 500 + i)).to(dev) for i, n in enumerate(MIXED)]
            ys = [torch.empty(n, dtype=torch.float16, device=dev) for n in MIXED]
            torch.cuda.synchronize()
            dist.barrier()
            for i, (part, y) in enumerate(zip(parts, ys)):
                if rank == world - 1:
                    torch.cuda._sleep(20000 + 15000 * (i % 4))
                ar(part, y)
            torch.cuda.synchronize()
            out_q.put((rank, "ok", ([y.cpu().numpy() for y in ys], ops.device_status(rank, clear=True))))
            dist.barrier()
        elif scenario == "sums":
            results = []
            for step, n in enumerate(SIZES * 2):
                part = torch.from_numpy(_partial(rank, n, step)).to(dev)
                y16 = torch.empty(n, dtype=torch.float16, device=dev)
                y32 = torch.empty(n, dtype=torch.float32, device=dev)
                ar(part, y16)
                ar(part, y32)
                torch.cuda.synchronize()
                results.append((n, step, y16.cpu().numpy(), y32.cpu().numpy()))
            # graph: three calls captured, replayed with fresh partials
            n = 5120
            part = torch.empty(n, dtype=torch.float32, device=dev)
            ys = [torch.empty(n, dtype=torch.float16, device=dev) for _ in range(3)]
            s = torch.cuda.Stream(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for y in ys:
                    ar(part, y)
            graph_results = []
            for step in range(100, 104):
                part.copy_(torch.from_numpy(_partial(rank, n, step)))
                torch.cuda.synchronize()
                with torch.cuda.stream(s):
                    g.replay()
                s.synchronize()
                graph_results.append((step, [y.cpu().numpy() for y in ys]))
            del g
            dist.barrier()
            out_q.put((rank, "ok", (results, graph_results)))
        else:  # "timeout": rank 1 never calls; rank 0's call gives up
            st = 0
            t = 0.0
            if rank == 0:
                part = torch.zeros(64, dtype=torch.float32, device=dev)
                y = torch.empty(64, dtype=torch.float16, device=dev)
                ops.device_status(rank, clear=True)
                t0 = time.time()
                ar(part, y)
                torch.cuda.synchronize()
                t = time.time() - t0
                st = ops.device_status(rank, clear=True)
            dist.barrier()
            out_q.put((rank, "ok", (st, t)))
        ar.close()
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


def _run(world, scenario):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, scenario)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 240
    while len(got) < world and time.time() < deadline:
        try:
            r, status, payload = q.get(timeout=10)
        except Exception:
            continue
        assert status == "ok", payload
        got[r] = payload
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert len(got) == world
    return got


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_allreduce_sums_exactly(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    got = _run(world, "sums")
    for r in range(world):
        results, graph_results = got[r]
        for n, step, y16, y32 in results:
            ref = _expected(world, n, step)
            np.testing.assert_array_equal(y32, ref)
            np.testing.assert_array_equal(y16.view(np.uint16), ref.astype(np.float16).view(np.uint16))
        for step, ys in graph_results:
            ref = _expected(world, 5120, step).astype(np.float16)
            for y in ys:
                np.testing.assert_array_equal(y.view(np.uint16), ref.view(np.uint16))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_allreduce_mixed_sizes_unsynchronized(world):
    """Grids of 148, 3, 40 and 1 chunks interleaved: every call's chunks share
    one epoch and parity, so a rank running ahead never stores into a slot a
    slower rank is still summing."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    got = _run(world, "mixed")
    for r in range(world):
        ys, status = got[r]
        assert status == 0
        for i, (n, y) in enumerate(zip(MIXED, ys)):
            ref = _expected(world, n, 500 + i).astype(np.float16)
            np.testing.assert_array_equal(y.view(np.uint16), ref.view(np.uint16), err_msg=f"call {i} (n={n})")


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_fused_row_parallel_matmul_equals_two_kernels(world):
    """qw_allreduce_matmul == qw_quantized_matmul (fp32) + qw_allreduce_sum,
    bit for bit, and the same on every rank.  World size 1 runs the fused
    epilogue against itself (each CTA flags and then reads its own tiles),
    on a one-GPU machine."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    got = _run(world, "matmul")
    for r in range(world):
        results, graph_results, status = got[r]
        assert status == 0
        for (i, dtype, y, ref), (_, _, y0, _) in zip(results, got[0][0]):
            np.testing.assert_array_equal(y.view(np.uint8), ref.view(np.uint8), err_msg=f"case {MATMULS[i]} {dtype}")
            np.testing.assert_array_equal(y.view(np.uint8), y0.view(np.uint8), err_msg=f"rank {r} vs 0, {MATMULS[i]}")
            assert np.isfinite(y.astype(np.float32)).all()
        for step, (ys, refs) in enumerate(graph_results):
            np.testing.assert_array_equal(ys[0].view(np.uint16), refs[0].view(np.uint16), err_msg=f"replay {step}")
            np.testing.assert_array_equal(ys[2].view(np.uint16), refs[1].view(np.uint16), err_msg=f"replay {step}")
            ref = _expected(world, 5120, 200 + step).astype(np.float16)
            np.testing.assert_array_equal(ys[1].view(np.uint16), ref.view(np.uint16), err_msg=f"replay {step}")


@pytest.mark.parametrize("world", [1, 2, 4])
def test_fused_matmul_interleaved_unsynchronized(world):
    """Fused matmuls (chunks = row tiles) and plain sums (chunks = CTAs of a
    size-dependent grid) share the communicator's epochs and parities."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    got = _run(world, "matmul_mixed")
    n = len(MATMULS)
    for r in range(world):
        refs, outs, status = got[r]
        assert status == 0
        for rep in range(2):
            for i in range(n):
                y = outs[2 * (rep * n + i)]
                np.testing.assert_array_equal(y.view(np.uint16), refs[i].view(np.uint16),
                                              err_msg=f"rank {r} pass {rep} matmul {MATMULS[i]}")
                s = outs[2 * (rep * n + i) + 1]
                ref = _expected(world, MIXED[i], 700 + i).astype(np.float16)
                np.testing.assert_array_equal(s.view(np.uint16), ref.view(np.uint16), err_msg=f"sum {i}")


def test_fused_matmul_absent_peer_times_out(cuda_dev):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    got = _run(2, "matmul_timeout")
    st, t = got[0]
    assert st != 0
    assert 1.5 < t < 30


def test_absent_peer_times_out(cuda_dev):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    got = _run(2, "timeout")
    st, t = got[0]
    assert st != 0  # QW status word: a bounded wait ran out
    assert 1.5 < t < 30
