"""The one-shot peer allreduce (qw_allreduce_sum) on P GPUs, one process per
GPU: every rank gets the fp32 partials summed in rank order, bit for bit the
float32 sum numpy forms in the same order (and its fp16 rounding); sizes that
are and are not multiples of the 4-float vector; repeated calls, eager and
replayed from a CUDA graph (the epoch advances on the device); calls of
different sizes (so different grids and chunk boundaries) issued back to back
with no host synchronization while one rank starts each call late; and a
rank whose peer never calls gives up after the bounded wait with a timeout
status instead of hanging.  Needs at least 2 GPUs (skipped otherwise); NVLS off."""
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
        ar = tp.PeerAllreduce(max(SIZES + MIXED))
        if scenario == "mixed":
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


def test_absent_peer_times_out(cuda_dev):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    got = _run(2, "timeout")
    st, t = got[0]
    assert st != 0  # QW status word: a bounded wait ran out
    assert 1.5 < t < 30
