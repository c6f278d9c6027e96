"""Tensor-parallel stack logic on CPU: two gloo ranks, each running its shard
of a (down-scaled) linear stack through the oracle, against the unsharded
stack.  Also a host-side failure case: a rank that dies before the collective
must not leave its peer hanging; and the peer allreduce's host protocol
(handle exchange, collective teardown) against a fake library.  No GPU."""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from qw_b200 import synth, tp
from tests.conftest import rel_err

DIMS = tp.StackDims(hidden=256, q_out=384, kv_out=64, inter=512, vocab=1000)
LAYERS = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    layers = []
    for l in range(LAYERS):
        d = {}
        for lin in DIMS.linears():
            w = synth.weight_fp16(lin.N, lin.K, seed=7, layer=l, tid=lin.tid, std=lin.K ** -0.5)
            d[lin.name] = oracle.quantize(w)
        layers.append(d)
    lm = DIMS.lm_head()
    lm_w = oracle.quantize(synth.weight_fp16(lm.N, lm.K, seed=7, layer=99, tid=lm.tid))
    return layers, lm_w


def _oracle_mm(x, w, out_f32):
    y, y32 = oracle.quantized_matmul(x, *w, want_f32=True)
    return y32 if out_f32 else y


def _oracle_swiglu(x, w):
    return oracle.quantized_matmul_swiglu(x, *tp.gate_up_halves(w))


def _reference_logits(x):
    layers, lm_w = _weights()
    stack = tp.LinearStack(layers, lm_w, 1, 0, _oracle_mm, None, None, DIMS, swiglu=_oracle_swiglu)
    return stack.forward(x)


def _rank_main(rank, world, port, x, out_q, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        layers, lm_w = _weights()
        lins = {l.name: l for l in DIMS.linears()}
        mine = [{n: tp.shard_linear(lins[n], *w, world, rank, DIMS) for n, w in d.items()} for d in layers]
        lm_mine = tp.shard_linear(DIMS.lm_head(), *lm_w, world, rank, DIMS)

        def allreduce(a):
            if rank == fail_rank:
                raise RuntimeError("injected rank failure")
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
            dist.all_reduce(t)
            return t.numpy()

        stack = tp.LinearStack(mine, lm_mine, world, rank, _oracle_mm, allreduce,
                               lambda a: a.astype(np.float16), DIMS, swiglu=_oracle_swiglu)
        t0 = time.time()
        logits = stack.forward(x)
        # greedy token over the vocabulary shards: this rank's keys, then the
        # int64 MAX exchange (the host-side statement of qw_allreduce_argmax)
        base = tp.column_shard_rows(DIMS.lm_head(), world, rank, DIMS)[0][0]
        keys = torch.from_numpy(np.ascontiguousarray(tp.signed_keys(tp.greedy_keys(logits, base))))
        token = tp.exchange_greedy_keys(keys).numpy()
        out_q.put((rank, "ok", (logits, token), time.time() - t0))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        out_q.put((rank, "error", repr(e), 0.0))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    x = synth.activations(3, DIMS.hidden, seed=5)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, x, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + 120
    while len(results) < world and time.time() < deadline:
        try:
            r, status, payload, dt = q.get(timeout=5)
            results[r] = (status, payload)
        except Exception:
            pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return x, results


def test_column_and_row_shards_reassemble():
    lins = DIMS.linears()
    for lin in lins:
        w = synth.weight_fp16(lin.N, lin.K, seed=1)
        wq, s, b = oracle.quantize(w)
        shards = [tp.shard_linear(lin, wq, s, b, 2, r, DIMS) for r in range(2)]
        for sh in shards:
            assert sh[0].shape == (tp.shard_shape(lin, 2)[0], tp.shard_shape(lin, 2)[1] // 8)
        x = synth.activations(2, lin.K, seed=2)
        if lin.row_parallel:
            k0, k1 = tp.row_shard_cols(lin.K, 2, 0)
            parts = [oracle.quantized_matmul(x[:, slice(*tp.row_shard_cols(lin.K, 2, r))], *shards[r], want_f32=True)[1]
                     for r in range(2)]
            full = oracle.quantized_matmul(x, wq, s, b, want_f32=True)[1]
            assert rel_err(parts[0] + parts[1], full) < 1e-5
        else:
            outs = [oracle.quantized_matmul(x, *shards[r]) for r in range(2)]
            full = oracle.quantized_matmul(x, wq, s, b)
            np.testing.assert_array_equal(tp.gather_columns(outs, lin, DIMS).view(np.uint16), full.view(np.uint16))


def test_row_shards_keep_groups_whole():
    with pytest.raises(ValueError):
        tp.row_shard_cols(64 * 3, 2, 0)  # 3 groups do not split over 2 ranks
    assert tp.row_shard_cols(17408, 8, 7) == (15232, 17408)


def test_two_rank_stack_matches_unsharded():
    x, results = _run(2)
    assert set(results) == {0, 1}, results
    ref = _reference_logits(x)
    shards, tokens = [], []
    for r in range(2):
        status, payload = results[r]
        assert status == "ok", payload
        shards.append(payload[0])
        tokens.append(payload[1])
    full = tp.gather_columns(shards, DIMS.lm_head(), DIMS)
    assert rel_err(full.astype(np.float32), ref.astype(np.float32)) <= 1e-2
    # both ranks hold the greedy token of the whole vocabulary
    want = oracle.topk(full, 1)[0][:, 0]
    for t in tokens:
        np.testing.assert_array_equal(t, want)


def _greedy_rank(rank, world, port, logits, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        n = logits.shape[1] // world
        keys = tp.greedy_keys(logits[:, rank * n:(rank + 1) * n], rank * n)
        token = tp.exchange_greedy_keys(torch.from_numpy(np.ascontiguousarray(tp.signed_keys(keys))))
        out_q.put((rank, "ok", token.numpy()))
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_greedy_token_exchange_ties_and_signs(world):
    """The (value, index) key exchange over gloo: equal maxima in different
    shards go to the lower global index, +0 outranks -0, an all-negative row
    and a row whose maximum sits in the last shard.  Every rank gets the
    argmax of the whole row."""
    rng = np.random.default_rng(3)
    N = 256 * world
    lg = (rng.standard_normal((6, N)) * 3).astype(np.float16)
    lg[0, 5] = lg[0, N - 7] = np.float16(30)           # tie across the first and last shard
    lg[1, :] = np.float16(0)
    lg[1, 3] = np.float16(-0.0)                          # index 0 holds +0: the answer
    lg[2, :] = -np.abs(lg[2, :]) - np.float16(1)          # all negative
    lg[3, N - 1] = np.float16(60)                        # the very last column
    lg[4, 256] = lg[4, 257] = np.float16(40)             # tie inside one shard
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_greedy_rank, args=(r, world, port, lg, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 120
    while len(got) < world and time.time() < deadline:
        try:
            r, status, payload = q.get(timeout=5)
            assert status == "ok", payload
            got[r] = payload
        except Exception as e:  # noqa: BLE001
            if isinstance(e, AssertionError):
                raise
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    want = oracle.topk(lg, 1)[0][:, 0]
    assert list(want[:5]) == [5, 0, int(np.argmax(lg[2])), N - 1, 256]
    assert len(got) == world
    for r in range(world):
        np.testing.assert_array_equal(got[r], want)


def test_failed_rank_does_not_hang_its_peer():
    """Rank 1 raises before its first allreduce; rank 0's collective must end
    with an error within the process-group timeout instead of waiting forever."""
    t0 = time.time()
    _, results = _run(2, fail_rank=1)
    assert results.get(1, ("", ""))[0] == "error"
    assert results.get(0, ("", ""))[0] == "error", results.get(0)
    assert time.time() - t0 < 100


# ------------------------------------------------- peer allreduce host protocol
class _FakeAllreduceLib:
    """Stands in for libqwqmm's qw_allreduce_* entry points (no GPU): each
    rank's IPC handle is 64 bytes of (rank + 1), and calls are logged."""

    def __init__(self, log):
        self.log = log

    def qw_allreduce_init(self, world, rank, max_elems, comm_ref, handle):
        import ctypes
        comm_ref._obj.value = 1000 + rank
        ctypes.memmove(handle, bytes([rank + 1]) * 64, 64)
        self.log.append(("init", world, rank, max_elems))
        return 0

    def qw_allreduce_connect(self, comm, blob):
        self.log.append(("connect", bytes(blob)))
        return 0

    def qw_allreduce_destroy(self, comm):
        self.log.append(("destroy", time.time()))
        return 0


def _protocol_rank(rank, world, port, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    from qw_b200 import _lib
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        log = []
        fake = _FakeAllreduceLib(log)
        _lib.load = lambda: fake                          # the fake library
        torch.cuda.current_device = lambda: 0             # no device here
        torch.cuda.synchronize = lambda *a, **k: log.append(("sync",))
        ar = tp.PeerAllreduce(4096)
        if rank == 0:
            time.sleep(1.5)  # the other ranks reach close first
        entered = time.time()
        ar.close()
        ar.close()  # a second close does nothing
        out_q.put((rank, "ok", (log, entered)))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        out_q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_host_protocol():
    """PeerAllreduce's host side over gloo with a fake library: every rank
    connects with all ranks' handles in rank order, and no rank frees its
    buffer (destroy) before every rank has reached close and synchronized."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_protocol_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 120
    while len(got) < world and time.time() < deadline:
        try:
            r, status, payload = q.get(timeout=5)
        except Exception:
            continue
        assert status == "ok", payload
        got[r] = payload
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert len(got) == world
    handles = b"".join(bytes([r + 1]) * 64 for r in range(world))
    last_entry = max(entered for _, entered in got.values())
    for r, (log, _) in got.items():
        kinds = [e[0] for e in log]
        assert kinds == ["init", "connect", "sync", "destroy"], kinds
        assert log[0] == ("init", world, r, 4096)
        assert log[1][1] == handles
        assert log[3][1] >= last_entry  # freed only after every rank reached close
