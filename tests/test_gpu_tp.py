"""Tensor-parallel linear stack on P GPUs, the o/down partial sums exchanged
by NCCL (fp32 allreduce, then a cast), by the library's one-shot peer
allreduce (qw_allreduce_sum, fp16 rounding fused), or inside the o/down
matmul itself (qw_allreduce_matmul: the decode kernel's epilogue for up to
16 rows, the matmul and the allreduce kernel above).

Checked two ways: against the same stack unsharded on one GPU (isolates the
sharding and the allreduce: only fp32 summation order differs), and against
the unsharded CPU oracle.  Both bounds are the per-op TOL scaled for the
chain: 13 quantized matmuls feed each other through fp16 activations and
SwiGLU products, and the prefill path (M >= 17) multiplies fp16-rounded
dequantized weights, so the per-op differences accumulate along the chain.
Needs at least 2 GPUs (skipped otherwise); one process per GPU, NVLS off,
short process-group timeout."""
import os
import socket
import time

import numpy as np
import pytest
import torch

import oracle
from qw_b200 import synth, tp
from tests.conftest import TOL, rel_err

pytestmark = pytest.mark.gpu

DIMS = tp.StackDims(hidden=1024, q_out=1536, kv_out=256, inter=2048, vocab=4096)
LAYERS = 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights():
    layers = []
    for l in range(LAYERS):
        layers.append({lin.name: oracle.quantize(synth.weight_fp16(lin.N, lin.K, seed=3, layer=l, tid=lin.tid,
                                                                   std=lin.K ** -0.5))
                       for lin in DIMS.linears()})
    lm = DIMS.lm_head()
    return layers, oracle.quantize(synth.weight_fp16(lm.N, lm.K, seed=3, layer=99, tid=lm.tid))


def _rank_main(rank, world, port, x, out_q, mode="nccl"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    import qw_b200
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        layers, lm_w = _weights()
        lins = {l.name: l for l in DIMS.linears()}

        def to_dev(w):
            wq, s, b = w
            return (torch.from_numpy(np.ascontiguousarray(wq).view(np.int32)).to(dev),
                    torch.from_numpy(np.ascontiguousarray(s)).to(dev), torch.from_numpy(np.ascontiguousarray(b)).to(dev))

        mine = [{n: to_dev(tp.shard_linear(lins[n], *w, world, rank, DIMS)) for n, w in d.items()} for d in layers]
        lm_mine = to_dev(tp.shard_linear(DIMS.lm_head(), *lm_w, world, rank, DIMS))

        def mm(xx, w, out_f32):
            return qw_b200.quantized_matmul(xx, *w, out_dtype=torch.float32 if out_f32 else torch.float16)

        rowpar = None
        if mode in ("peer", "fused"):
            ar = tp.PeerAllreduce(64 * DIMS.hidden)

            def allreduce(t):  # fp32 partials in, fp16 sums out
                return ar(t, torch.empty(t.shape, dtype=torch.float16, device=t.device))
        else:
            def allreduce(t):
                dist.all_reduce(t)
                return t

        def swiglu(xx, w):
            return qw_b200.quantized_matmul_swiglu(xx, *[t for half in tp.gate_up_halves(w) for t in half])

        if mode == "fused":
            def rowpar(xx, w):
                return ar.matmul(xx, w, torch.empty(xx.shape[0], w[0].shape[0], dtype=torch.float16, device=dev))

        stack = tp.LinearStack(mine, lm_mine, world, rank, mm, allreduce, lambda t: t.half(), DIMS, swiglu=swiglu,
                               rowpar=rowpar)
        torch.cuda.synchronize()
        for M in (1, 16, 64):
            y = stack.forward(torch.from_numpy(x[:M]).to(dev))
            torch.cuda.synchronize()
            out_q.put((rank, M, "ok", y.cpu().numpy()))
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, -1, "error", repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["nccl", "peer", "fused"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_stack_matches_oracle(world, mode):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    x = synth.activations(64, DIMS.hidden, seed=9)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, x, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 300
    while len(got) < 3 * world and time.time() < deadline:
        try:
            r, M, status, payload = q.get(timeout=10)
        except Exception:
            continue
        assert status == "ok", payload
        got[(r, M)] = payload
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert len(got) == 3 * world
    layers, lm_w = _weights()

    def omm(xx, w, out_f32):
        """The oracle in the arithmetic of the kernel that runs: fp32-formed
        weights for at most 16 rows, the fp16 dequantized weights above."""
        if xx.shape[0] <= 16:
            y, y32 = oracle.quantized_matmul(xx, *w, want_f32=True)
            return y32 if out_f32 else y
        y64 = xx.astype(np.float64) @ oracle.dequantize(*w).astype(np.float64).T
        return y64.astype(np.float32) if out_f32 else y64.astype(np.float16)

    import qw_b200
    dev = torch.device("cuda", 0)

    def to_dev(w):
        wq, s_, b_ = w
        return (torch.from_numpy(np.ascontiguousarray(wq).view(np.int32)).to(dev),
                torch.from_numpy(np.ascontiguousarray(s_)).to(dev), torch.from_numpy(np.ascontiguousarray(b_)).to(dev))

    def gmm(xx, w, out_f32):
        return qw_b200.quantized_matmul(xx, *w, out_dtype=torch.float32 if out_f32 else torch.float16)

    def gswiglu(xx, w):
        return qw_b200.quantized_matmul_swiglu(xx, *[t for half in tp.gate_up_halves(w) for t in half])

    def oswiglu(xx, w):
        g, u = tp.gate_up_halves(w)
        return oracle.swiglu(omm(xx, g, False), omm(xx, u, False))

    one_gpu = tp.LinearStack([{n: to_dev(w) for n, w in d.items()} for d in layers], to_dev(lm_w), 1, 0, gmm,
                             None, None, DIMS, swiglu=gswiglu)
    ref_stack = tp.LinearStack(layers, lm_w, 1, 0, omm, None, None, DIMS, swiglu=oswiglu)
    n_ops = 4 * LAYERS + 1
    for M in (1, 16, 64):
        full = tp.gather_columns([got[(r, M)] for r in range(world)], DIMS.lm_head(), DIMS).astype(np.float32)
        single = one_gpu.forward(torch.from_numpy(x[:M]).to(dev)).float().cpu().numpy()
        # only the fp32 partial-sum order differs; the fp16 rounding flips it
        # causes propagate through the chain's SwiGLU products like the
        # per-op differences against the oracle below
        assert rel_err(full, single) <= TOL * np.sqrt(n_ops), (world, M)
        ref = ref_stack.forward(x[:M]).astype(np.float32)
        assert rel_err(full, ref) <= TOL * np.sqrt(n_ops), (world, M)


ARGMAX_VOCAB, ARGMAX_K = 32768, 512  # one 512-wide chunk: every row's logit is one CTA's, whatever the shard


def _argmax_rank(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch.distributed as dist
    import qw_b200
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        lm = tp.StackDims(hidden=ARGMAX_K, vocab=ARGMAX_VOCAB).lm_head()
        full_np = oracle.quantize(synth.weight_fp16(lm.N, lm.K, seed=4, layer=99, tid=lm.tid))
        full = tuple(torch.from_numpy(np.ascontiguousarray(a).view(np.int32) if a.dtype == np.uint32 else a).to(dev)
                     for a in full_np)
        n = lm.N // world
        mine = tuple(t[rank * n:(rank + 1) * n].contiguous() for t in full)
        ar = tp.PeerAllreduce(64)
        x_all = torch.from_numpy(synth.activations(20, lm.K, seed=8)).to(dev)
        for M in (1, 4, 16, 20):
            x = x_all[:M].contiguous()
            logits = torch.empty(M, n, dtype=torch.float16, device=dev) if M > 16 else None
            idx = ar.argmax(x, mine, rank * n, logits=logits)
            full_logits = torch.empty(M, lm.N, dtype=torch.float16, device=dev) if M > 16 else None
            one = qw_b200.quantized_matmul_argmax(x, *full, logits=full_logits)
            torch.cuda.synchronize()
            out_q.put((rank, M, "ok", ((idx.to(torch.int64) & 0xFFFFFFFF).cpu().numpy(), one.cpu().numpy())))
        # replayed from a CUDA graph: the exchange's epoch advances on the device
        x = x_all[:1].contiguous()
        idx = torch.empty(1, dtype=torch.int32, device=dev)
        s = torch.cuda.Stream(dev)
        with torch.cuda.stream(s):
            ar.argmax(x, mine, rank * n, idx=idx)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ar.argmax(x, mine, rank * n, idx=idx)
        replays = []
        for i in range(3):
            x.copy_(x_all[i + 1:i + 2])
            torch.cuda.synchronize()
            with torch.cuda.stream(s):
                g.replay()
            s.synchronize()
            replays.append(((idx.to(torch.int64) & 0xFFFFFFFF).cpu().numpy(),
                            qw_b200.quantized_matmul_argmax(x, *full).cpu().numpy()))
        del g
        out_q.put((rank, -2, "ok", replays))
        status = qw_b200.device_status(rank, clear=False)
        ar.close()
        out_q.put((rank, -3, "ok", status))
    except Exception as e:  # noqa: BLE001
        out_q.put((rank, -1, "error", repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_greedy_token_matches_one_gpu(world):
    """qw_allreduce_argmax over vocabulary shards returns, on every rank, the
    greedy token one GPU holding the whole LM head returns (fused decode
    epilogue for M <= 16, logits and a row reduction for M = 20), also when
    replayed from a CUDA graph.  World size 1 runs the exchange kernel
    against itself, on a one-GPU machine."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_argmax_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 300
    while len(got) < 6 * world and time.time() < deadline:
        try:
            r, M, status, payload = q.get(timeout=10)
        except Exception:
            continue
        assert status == "ok", payload
        got[(r, M)] = payload
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert len(got) == 6 * world
    for r in range(world):
        for M in (1, 4, 16, 20):
            idx, one = got[(r, M)]
            np.testing.assert_array_equal(idx, one, err_msg=f"rank {r} M={M}")
        for idx, one in got[(r, -2)]:
            np.testing.assert_array_equal(idx, one)
        assert got[(r, -3)] == 0
