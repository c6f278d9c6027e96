#!/usr/bin/env python
"""Benchmark of the 4-bit affine group-64 quantized matmul hot path.

Headline (BASELINE metric "4-bit qmatmul HBM GB/s & % peak at M=1/16; 27B
linear-stack tok/s"): decode tokens/s of the 64-layer Qwen 27B linear stack at
M=1 (q|k|v 5120->8192, o 6144->5120, gate|up 5120->34816, down 17408->5120 per
layer, then lm_head 5120->151936 and the greedy token over the vocabulary),
synthetic seeded weights quantized on the GPU by the library's own quantizer.  The MLP's gate|up projection runs with
its SwiGLU activation fused (qw_quantized_matmul_swiglu), so down consumes
silu(gate) * up as in the model.  One step = one token through the stack.

  value   device-resident inputs, the step captured once as a CUDA graph of
          the library's launches (programmatic dependent launch between them)
  e2e     the same step through the public C ABI call by call (qw_quantized_matmul
          and qw_quantized_matmul_swiglu via ctypes), x copied from pinned host
          memory before and the step's greedy token read back after, every step
Extra keys report the single-matrix qmv (M=1) and verify qmm (M=16) GB/s with
L2 defeated by rotating weight copies, and the M=16 stack.

With torchrun (N > 1) the stack is tensor-parallel: q/k/v/gate/up/lm_head
column-sharded, o/down row-sharded.  With the library's peer exchange (the
default) o and down are qw_allreduce_matmul calls: each 128-row tile's fp32
products go to every rank over NVLink from the decode kernel's epilogue and
are summed there, one launch per projection (`--tp-allreduce nccl`: the
matmul, ncclAllReduce and a cast, for comparison).  Rank 0 prints
one JSON line.  `--impl reference` times the reference's CPU path (the oracle
restatement of MLX's affine quantized_matmul; the reference itself cannot be
built here) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from qw_b200 import synth, tp  # noqa: E402

METRIC = "4-bit qmatmul HBM GB/s & % peak at M=1/16; 27B linear-stack tok/s"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def profile_traffic(key):
    """DRAM bytes per launch from a committed ncu summary (profiles/traffic.txt)."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 2 and parts[0] == key:
                return float(parts[1])
    except OSError:
        pass
    return None


# ----------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = str(index)
        self.proc = None
        try:  # nvidia-smi numbers GPUs differently from CUDA_VISIBLE_DEVICES; use the UUID
            import torch
            u = str(torch.cuda.get_device_properties(int(index)).uuid)
            self.index = u if u.startswith("GPU-") else "GPU-" + u
        except Exception:
            pass

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.index, f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------ the GPU arm
def make_weights(torch, qw, N, K, seed, dev, group_size=64, bits=4):
    """N x K fp16 ~ N(0, 0.02), quantized on the GPU; returns (wq, scales, biases)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    wq = torch.empty(N, K * bits // 32, dtype=torch.int32, device=dev)
    s = torch.empty(N, K // group_size, dtype=torch.float16, device=dev)
    b = torch.empty(N, K // group_size, dtype=torch.float16, device=dev)
    rows = max(1, (1 << 27) // K)  # quantize in slabs of ~256 MB of fp16
    for r0 in range(0, N, rows):
        r1 = min(N, r0 + rows)
        w = (torch.randn(r1 - r0, K, generator=g, device=dev, dtype=torch.float32) * 0.02).half()
        wq_s, s_s, b_s = qw.quantize_weights(w, group_size=group_size, bits=bits)
        wq[r0:r1].copy_(wq_s)
        s[r0:r1].copy_(s_s)
        b[r0:r1].copy_(b_s)
        del w, wq_s, s_s, b_s
    return wq, s, b


def build_stack(torch, qw, P, rank, layers, dev):
    ws = []
    for l in range(layers):
        d = {}
        for lin in synth.layer_linears():
            N, K = tp.shard_shape(lin, P)
            d[lin.name] = make_weights(torch, qw, N, K, seed=(l * 16 + lin.tid) * 64 + rank, dev=dev)
        ws.append(d)
    N, K = tp.shard_shape(synth.LM_HEAD, P)
    lm = make_weights(torch, qw, N, K, seed=(99 * 16 + 9) * 64 + rank, dev=dev)
    return ws, lm


class StackRunner:
    """Fixed buffers + the per-step launch sequence, for graph capture and eager e2e.

    Per layer: qkv, o, the MLP's gate and up projections with SwiGLU fused
    (qw_quantized_matmul_swiglu over the two row halves of the rank's gate_up
    shard), down; then lm_head and the greedy token of each row (under tensor
    parallelism over every rank's vocabulary shard).  chain=False issues one C-ABI call per
    linear (the drop-in path); chain=True hands each run of plain matmuls
    with nothing in between (down of one layer with qkv and o of the next on
    one GPU; qkv+o between allreduces under tensor parallelism) to
    qw_quantized_matmul_chain."""

    def __init__(self, torch, qw, ws, lm, M, P, group, chain=False, ar=None):
        self.torch, self.qw, self.ws, self.lm, self.M, self.P, self.group = torch, qw, ws, lm, M, P, group
        self.ar = ar  # tp.PeerAllreduce, or None for NCCL
        self.chain = chain and M <= 16
        dev = lm[0].device
        H = synth.HIDDEN
        f16, f32 = torch.float16, torch.float32
        self.h = torch.randn(M, H, device=dev).half()
        nq = tp.shard_shape(synth.layer_linears()[0], P)[0]
        ngu = tp.shard_shape(synth.layer_linears()[2], P)[0]
        self.qkv = torch.empty(M, nq, dtype=f16, device=dev)
        self.attn = torch.empty(M, synth.Q_OUT // P, dtype=f16, device=dev)
        self.gate = torch.empty(M, ngu // 2, dtype=f16, device=dev)  # silu(gate) * up, down's input
        self.halves = [tuple(t for half in tp.gate_up_halves(w["gate_up"]) for t in half) for w in ws]
        self.part = torch.empty(M, H, dtype=f32, device=dev)
        self.o = torch.empty(M, H, dtype=f16, device=dev)
        self.logits = torch.empty(M, lm[0].shape[0], dtype=f16, device=dev)
        # the step's result: the greedy token of every row over the whole vocabulary
        self.token = torch.empty(M, dtype=torch.int32, device=dev)
        self.vocab_base = (torch.distributed.get_rank(group) if P > 1 else 0) * lm[0].shape[0]
        # this library's kernels per step: per layer 4 matmuls (under tensor
        # parallelism with the peer exchange, o and down sum over the ranks in
        # their own epilogue for M <= 16, else an allreduce kernel follows
        # each); then lm_head with the greedy token: the fused epilogue and its
        # finalize (1 GPU), the matmul and the peer exchange kernel, or the
        # matmul alone (NCCL: the keys and the all-reduce are torch's and
        # NCCL's kernels)
        L = len(ws)
        if P == 1:
            self.launches_per_step = 4 * L + 2
        elif ar is not None:
            self.launches_per_step = (4 if M <= 16 else 6) * L + 2
        else:
            self.launches_per_step = 4 * L + 1
        if self.chain:
            self._build_segments()

    def _build_segments(self):
        """The step as actions: ("chain", ops) runs of plain matmuls,
        ("swiglu", layer) the fused MLP input projections, ("reduce", dst)
        the tensor-parallel allreduce of the fp32 partials into dst."""
        q_view = self.qkv[:, : self.attn.shape[1]]   # row-strided view: no copy
        acts, cur = [], []

        def flush():
            if cur:
                acts.append(("chain", list(cur)))
                cur.clear()

        for l, w in enumerate(self.ws):
            cur.append((self.h, *w["qkv"], self.qkv))
            if self.P == 1:
                cur.append((q_view, *w["o"], self.o))
            else:
                cur.append((q_view, *w["o"], self.part))
                flush()
                acts.append(("reduce", self.o))
            flush()
            acts.append(("swiglu", l))
            if self.P == 1:
                cur.append((self.gate, *w["down"], self.h))
            else:
                cur.append((self.gate, *w["down"], self.part))
                flush()
                acts.append(("reduce", self.h))
        flush()
        acts.append(("token", None))
        self.actions = acts
        self.launches_per_step = (sum((len(a[1]) + 23) // 24 for a in acts if a[0] == "chain")
                                  + sum(1 for a in acts if a[0] == "swiglu")
                                  + sum(1 for a in acts if a[0] == "reduce" and self.ar is not None)
                                  + (2 if self.P == 1 or self.ar is not None else 1))

    def _mm(self, x, w, out):
        self.qw.quantized_matmul(x, w[0], w[1], w[2], out=out)

    def _reduce(self, out16):
        """out16 = fp16(sum over ranks of self.part)."""
        if self.ar is not None:
            self.ar(self.part, out16)
        else:
            self.torch.distributed.all_reduce(self.part, group=self.group)
            out16.copy_(self.part)

    def _rowpar(self, x, w, out16):
        if self.P == 1:
            self._mm(x, w, out16)
        elif self.ar is not None:
            self.ar.matmul(x, w, out16)  # the sum over ranks fused (qw_allreduce_matmul)
        else:
            self._mm(x, w, self.part)
            self._reduce(out16)

    def _swiglu(self, x, l, out):
        self.qw.quantized_matmul_swiglu(x, *self.halves[l], out=out)

    def _token(self):
        """lm_head and the greedy token of each row over the whole vocabulary
        into self.token: fused into the decode kernel's epilogue on one GPU,
        qw_allreduce_argmax over the vocabulary shards with the peer exchange,
        or the shard's keys and an int64 MAX all-reduce with NCCL."""
        M = self.M
        logits = self.logits if M > 16 else None
        if self.P == 1:
            self.qw.quantized_matmul_argmax(self.h, *self.lm, logits=self.logits, idx=self.token)
        elif self.ar is not None:
            self.ar.argmax(self.h, self.lm, self.vocab_base, idx=self.token, logits=logits)
        else:
            self._mm(self.h, self.lm, self.logits)
            keys = tp.greedy_keys_torch(self.logits, self.vocab_base)
            self.token.copy_(tp.exchange_greedy_keys(keys, self.group))

    def step(self):
        if self.chain:
            for a in self.actions:
                if a[0] == "chain":
                    self.qw.quantized_matmul_chain(a[1])
                elif a[0] == "swiglu":
                    self._swiglu(self.o, a[1], self.gate)
                elif a[0] == "token":
                    self._token()
                else:
                    self._reduce(a[1])
            return
        M = self.M
        for l, w in enumerate(self.ws):
            self._mm(self.h, w["qkv"], self.qkv)
            if M == 1:
                attn = self.qkv[:, : self.attn.shape[1]]
            else:
                self.attn.copy_(self.qkv[:, : self.attn.shape[1]])
                attn = self.attn
            self._rowpar(attn, w["o"], self.o)
            self._swiglu(self.o, l, self.gate)
            self._rowpar(self.gate, w["down"], self.h)
        self._token()


def timed_graph(torch, runner, steps, warmup, stream, dist_on, sampler_index):
    """Capture one step as a CUDA graph and time `steps` replays (max over ranks)."""
    with torch.cuda.stream(stream):
        for _ in range(2):
            runner.step()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        runner.step()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            g.replay()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist_on:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(sampler_index) as cs:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(steps):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize()
    if dist_on:
        torch.distributed.barrier()
    ms = e0.elapsed_time(e1) / steps
    ms = reduce_max(torch, ms, dist_on)
    del g
    return ms, cs.summary()


def timed_e2e(torch, runner, steps, warmup, stream, dist_on):
    """Eager C-ABI calls; h2d of x from pinned memory and d2h of logits every step."""
    M = runner.M
    x_host = torch.randn(M, synth.HIDDEN).half().pin_memory()
    y_host = torch.empty(runner.token.shape, dtype=runner.token.dtype).pin_memory()

    def one():
        runner.h.copy_(x_host, non_blocking=True)
        runner.step()
        y_host.copy_(runner.token, non_blocking=True)  # the greedy token of the step

    with torch.cuda.stream(stream):
        for _ in range(warmup):
            one()
    stream.synchronize()
    if dist_on:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(steps):
            one()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = reduce_max(torch, e0.elapsed_time(e1) / steps, dist_on)
    return ms, x_host.numel() * 2, y_host.numel() * 4


def reduce_max(torch, v, dist_on):
    if not dist_on:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def kernel_microbench(torch, qw, M, N, K, dev, copies=8, iters=50, swiglu=False, group_size=64, bits=4):
    """One quantized matmul, rotating `copies` weight sets (> L2) between launches.
    swiglu=True runs the fused SwiGLU over the two row halves of each N-row set
    (N/2 outputs per row of x)."""
    sets = [make_weights(torch, qw, N, K, seed=7000 + i, dev=dev, group_size=group_size, bits=bits)
            for i in range(copies)]
    x = torch.randn(M, K, device=dev).half()
    y = torch.empty(M, N // 2 if swiglu else N, dtype=torch.float16, device=dev)
    if swiglu:
        calls = [tuple(t for half in tp.gate_up_halves(w) for t in half) for w in sets]
    s = torch.cuda.Stream(dev)

    def call(i):
        if swiglu:
            qw.quantized_matmul_swiglu(x, *calls[i % copies], out=y)
        else:
            w = sets[i % copies]
            qw.quantized_matmul(x, w[0], w[1], w[2], group_size=group_size, bits=bits, out=y)

    with torch.cuda.stream(s):
        for i in range(copies * 2):
            call(i)
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(copies):
            call(i)
    with torch.cuda.stream(s):
        g.replay()
    s.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(iters):
            g.replay()
        e1.record(s)
    s.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / (iters * copies)
    nbytes = (N * K * bits // 8 + 4 * N * (K // group_size) + 2 * M * K
              + 2 * M * (N // 2 if swiglu else N))  # codes, scales + biases, x, y (SwiGLU writes N/2)
    del g, sets
    torch.cuda.empty_cache()
    return us, nbytes / (us * 1e-6) / 1e9


def graph_time_us(torch, fn, dev, iters=20):
    """Device time of fn() per call, captured once in a CUDA graph of `iters` calls."""
    s = torch.cuda.Stream(dev)
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    s.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(iters):
            fn()
    with torch.cuda.stream(s):
        for _ in range(3):
            g.replay()
    s.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(reps):
            g.replay()
        e1.record(s)
    s.synchronize()
    del g
    return e0.elapsed_time(e1) * 1000.0 / (iters * reps)


def cpu_stack_rate(ws, lm, threads, passes=2):
    """The oracle (C, OpenMP, `threads` threads) over the whole stack's
    quantized weights copied to the host (the same bytes the GPU streams), M=1.
    Returns (GB/s, seconds of CPU work)."""
    import oracle

    def host(w):
        return (w[0].cpu().numpy().view(np.uint32), w[1].cpu().numpy(), w[2].cpu().numpy())

    mats = [host(l[n]) for l in ws for n in l] + [host(lm)]
    t_total, b_total = 0.0, 0
    for _ in range(passes):
        for wq, s, b in mats:
            N, K = wq.shape[0], wq.shape[1] * 8
            x = synth.activations(1, K, seed=1)
            t0 = time.perf_counter()
            oracle.quantized_matmul(x, wq, s, b, nthreads=threads)
            t_total += time.perf_counter() - t0
            b_total += synth.algorithmic_bytes(1, N, K)
    return b_total / t_total / 1e9, t_total


def run_ours(args):
    import torch
    import qw_b200 as qw

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist_on = world > 1
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if dist_on:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
        group = torch.distributed.group.WORLD
    P = world
    hbm_peak, tf_peak, peak_src = peaks()

    ws, lm = build_stack(torch, qw, P, rank, args.layers, dev)
    torch.cuda.synchronize()
    ar = None
    if dist_on and args.tp_allreduce == "peer":
        from qw_b200 import tp as tpm
        ar = tpm.PeerAllreduce(2048 * synth.HIDDEN, group=group)  # the largest row-parallel output
    stream = torch.cuda.Stream(dev)

    # value: one qw_quantized_matmul per linear (the drop-in path), the step
    # captured once as a CUDA graph with programmatic dependent launch
    runner = StackRunner(torch, qw, ws, lm, 1, P, group, chain=False, ar=ar)
    ms, clocks = timed_graph(torch, runner, args.steps, args.warmup, stream, dist_on, local)
    step_bytes = synth.stack_bytes(1, layers=args.layers) // P if P > 1 else synth.stack_bytes(1, layers=args.layers)
    tok_s = 1000.0 / ms
    launches = runner.launches_per_step
    e2e_ms, h2d, d2h = timed_e2e(torch, runner, args.steps, args.warmup, stream, dist_on)
    # the same step through qw_quantized_matmul_chain (runs of linears per cooperative launch)
    chained = StackRunner(torch, qw, ws, lm, 1, P, group, chain=True, ar=ar)
    ms_chain, _ = timed_graph(torch, chained, args.steps, args.warmup, stream, dist_on, local)
    chain_launches = chained.launches_per_step
    del chained

    extra = {"stack_m1_chain": {"tok_s": round(1000.0 / ms_chain, 2), "ms_per_step": round(ms_chain, 5),
                                "GBps_per_gpu": round(step_bytes / (ms_chain * 1e-3) / 1e9, 1),
                                "frac_hbm": round(step_bytes / (ms_chain * 1e-3) / 1e9 / hbm_peak, 4),
                                "launches_per_step": chain_launches,
                                "path": "qw_quantized_matmul_chain, CUDA graph"}}
    if not args.skip_extra:
        # verify-batch stacks (MTP M=4, DFlash2 block M=16): HBM-bound like M=1
        for Mv in (4, 16):
            rv = StackRunner(torch, qw, ws, lm, Mv, P, group, ar=ar)
            msv, _ = timed_graph(torch, rv, max(10, args.steps // 4), args.warmup, stream, dist_on, local)
            bv = synth.stack_bytes(Mv, layers=args.layers) // P
            extra[f"stack_m{Mv}"] = {"tok_s": round(Mv * 1000.0 / msv, 1), "ms_per_step": round(msv, 4),
                                     "GBps_per_gpu": round(bv / (msv * 1e-3) / 1e9, 1),
                                     "frac_hbm": round(bv / (msv * 1e-3) / 1e9 / hbm_peak, 4),
                                     "weight_reuse_vs_m1": Mv}
            del rv
        # prefill chunk (M=2048) through the same stack: tensor-bound (tcgen05)
        rp = StackRunner(torch, qw, ws, lm, 2048, P, group, ar=ar)
        msp, _ = timed_graph(torch, rp, 3, 3, stream, dist_on, local)
        fl = synth.stack_flops(2048, layers=args.layers) / P
        extra["stack_prefill_m2048"] = {"tok_s": round(2048 * 1000.0 / msp, 1), "ms_per_step": round(msp, 3),
                                        "TFLOPs_per_gpu": round(fl / (msp * 1e-3) / 1e12, 1),
                                        "frac_tensor_bf16_burst": round(fl / (msp * 1e-3) / 1e12 / tf_peak, 4),
                                        "frac_2250TF_nominal": round(fl / (msp * 1e-3) / 1e12 / 2250.0, 4)}
        del rp
        torch.cuda.empty_cache()
        if rank == 0 and P == 1:
            for M in (1, 4, 16):
                us, gbs = kernel_microbench(torch, qw, M, 17408, 5120, dev)
                extra[f"qmm_17408x5120_m{M}"] = {"us": round(us, 2), "GBps": round(gbs, 1),
                                                 "frac_hbm": round(gbs / hbm_peak, 4),
                                                 "frac_8TBps": round(gbs / 8000.0, 4)}
            # the per-tensor override configurations at decode: 4-bit groups of 128
            # (the decode kernel) and 8-bit groups of 64 (the tensor-core kernel)
            for bits, gsz in ((4, 128), (8, 64)):
                us, gbs = kernel_microbench(torch, qw, 1, 17408, 5120, dev, copies=4, group_size=gsz, bits=bits)
                extra[f"qmm_17408x5120_b{bits}g{gsz}_m1"] = {"us": round(us, 2), "GBps": round(gbs, 1),
                                                             "frac_hbm": round(gbs / hbm_peak, 4)}
            # the DFlash2 candidate step: lm_head at M=16 then the top 16 of each row
            xl = torch.randn(16, synth.HIDDEN, device=dev).half()
            lg = torch.empty(16, lm[0].shape[0], dtype=torch.float16, device=dev)
            us_mm = graph_time_us(torch, lambda: qw.quantized_matmul(xl, *lm, out=lg), dev)
            us_tk = graph_time_us(torch, lambda: qw.quantized_matmul_topk(xl, *lm, 16, logits=lg), dev)
            extra["lm_head_top16_m16"] = {"us": round(us_tk, 2), "matmul_only_us": round(us_mm, 2),
                                          "topk_us": round(us_tk - us_mm, 2)}
            # the MLP input: gate and up 17408 x 5120 each, SwiGLU fused, against
            # the unfused 34816-row matmul of the same weights
            for M in (1, 16):
                us_f, gbs_f = kernel_microbench(torch, qw, M, 2 * synth.INTER, synth.HIDDEN, dev, copies=4,
                                                swiglu=True)
                us_p, _ = kernel_microbench(torch, qw, M, 2 * synth.INTER, synth.HIDDEN, dev, copies=4)
                extra[f"swiglu_gate_up_m{M}"] = {"us": round(us_f, 2), "GBps": round(gbs_f, 1),
                                                 "frac_hbm": round(gbs_f / hbm_peak, 4),
                                                 "unfused_matmul_us": round(us_p, 2)}

    result = {
        "metric": METRIC,
        "value": round(tok_s, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "f16 activations, u4 weights, f32 accumulate",
        "data": "synthetic: x~N(0,1), W~N(0,0.02) fp16 quantized on GPU (affine, 4-bit, group 64)",
        "config": stack_config(args, world),
        "GBps_per_gpu": round(step_bytes / (ms * 1e-3) / 1e9, 1),
        "roofline": None,
        "e2e": {"value": round(1000.0 / e2e_ms, 2), "unit": "tok/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 5),
                "path": "qw_quantized_matmul per layer via ctypes, eager, pinned host x in / greedy token out"},
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
        # a kernel whose bounded wait ran out (a missing peer, a stalled pipeline)
        # leaves a code here; 0 means every wait of the run completed
        "device_status": qw.device_status(local, clear=False),
        "extra": extra,
    }
    achieved = step_bytes / (ms * 1e-3) / 1e9
    traffic = profile_traffic("qmm_skinny_m1_stack_step")
    traffic_note = "ncu DRAM bytes of one 1-GPU decode step"
    if traffic is not None and (P > 1 or args.layers != synth.LAYERS):
        # per rank: the 1-GPU 64-layer step's DRAM bytes in the proportion of
        # the rank's algorithmic bytes (every weight matrix is split evenly)
        traffic = traffic * step_bytes / synth.stack_bytes(1)
        traffic_note = (f"per rank: the 1-GPU {synth.LAYERS}-layer capture scaled by the rank's share of the "
                        f"algorithmic bytes ({args.layers} layers, 1/{P})")
    result["roofline"] = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                          "frac": round(achieved / hbm_peak, 4), "peak_source": peak_src,
                          "kernel": "qmm_skinny_kernel (every launch of the step)",
                          "traffic": None if traffic is None else round(traffic), "traffic_source": traffic_note}

    if rank == 0 and world == 1 and not args.skip_cpu:
        threads = os.cpu_count() or 1
        gbs, secs = cpu_stack_rate(ws, lm, threads)
        result["cpu_baseline"] = {
            "value": round(gbs * 1e9 / synth.stack_bytes(1, args.layers), 4), "unit": "tok/s", "cores": threads,
            "kind": "port", "GBps": round(gbs, 3),
            "sample": f"the whole {args.layers}-layer stack + lm_head at M=1, twice, through the C oracle (AVX2, OpenMP) "
                      f"({secs:.1f} s of CPU work) on the GPU's quantized weights copied to the host"}
    if dist_on:
        torch.distributed.barrier()
        if ar is not None:
            ar.close()
        torch.distributed.destroy_process_group()
    if rank == 0:
        benchmark_result_line("qw_b200_decode_stack_m1", 1, args.steps, ms * 1e-3 * args.steps)
        print(json.dumps(result), flush=True)


def benchmark_result_line(label, tokens_per_repetition, repetitions, elapsed_s):
    """The reference benchmark's result line (crates/runtime/benches/
    single_user_throughput.rs:126-131), on stderr so that stdout keeps the
    single JSON line.  The steps are timed as one bracketed region, so there
    is no per-step spread: stddev_seconds is nan.  context_tokens is 0: the
    linear stack has no attention context."""
    processed = tokens_per_repetition * repetitions
    print(f"BENCHMARK_RESULT label={label} context_tokens=0 tokens_per_repetition={tokens_per_repetition} "
          f"processed_tokens={processed} repetitions={repetitions} elapsed_seconds={elapsed_s:.6f} "
          f"mean_seconds={elapsed_s / repetitions:.6f} stddev_seconds=nan "
          f"tokens_per_second={processed / elapsed_s:.3f}", file=sys.stderr, flush=True)


def stack_config(args, world):
    """The workload description both arms print (identical, so the driver can
    compare the two lines)."""
    return {"workload": f"decode linear stack M=1, {args.layers} layers (qkv/o/gate_up+SwiGLU/down) + lm_head",
            "M": 1, "layers": args.layers, "hidden": synth.HIDDEN, "vocab": synth.VOCAB,
            "parallelism": ((f"tp{world}, o/down summed over ranks in the matmul epilogue (NVLink peer stores)"
                             if args.tp_allreduce == "peer" else f"tp{world}, nccl allreduce")
                            if world > 1 else "single"),
            "l2": "inputs larger than L2 (weights %.2f GB per step)" % (synth.stack_bytes(1, args.layers) / 1e9),
            "graph": "one CUDA graph per step, programmatic dependent launch"}


def run_reference(args):
    """The reference's CPU path (the oracle restatement of MLX's affine
    quantized_matmul) on the host cores: every step is one token through the
    whole stack, as the GPU arm's step is -- per layer q|k|v, o, gate|up with
    the SwiGLU activation on its two halves, down, then lm_head -- with one
    decoder layer's quantized weights used for all layers (one layer is 192 MB,
    so every layer still streams its weights from DRAM)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    import oracle
    threads = os.cpu_count() or 1
    lins = synth.layer_linears()
    mats = {lin.name: oracle.quantize(synth.weight_fp16(lin.N, lin.K, seed=lin.tid)) for lin in lins}
    lm = oracle.quantize(synth.weight_fp16(synth.LM_HEAD.N, synth.LM_HEAD.K, seed=synth.LM_HEAD.tid))
    xs = {K: synth.activations(1, K, seed=2) for K in {lin.K for lin in lins}}

    def step():
        for _ in range(args.layers):
            for lin in lins:
                y = oracle.quantized_matmul(xs[lin.K], *mats[lin.name], nthreads=threads)
                if lin.name == "gate_up":  # the MLP activation on the gate and up halves
                    oracle.swiglu(y[:, : lin.N // 2], y[:, lin.N // 2:])
        return oracle.quantized_matmul(xs[synth.HIDDEN], *lm, nthreads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    nbytes = synth.stack_bytes(1, args.layers)
    tok_s = args.steps / dt
    sample = (f"the whole {args.layers}-layer stack + lm_head per step (one token, M=1) through the C oracle "
              f"(AVX2, OpenMP, {threads} threads), SwiGLU on the gate_up halves; one layer's weights serve "
              f"every layer")
    out = {
        "impl": "reference", "metric": METRIC, "value": round(tok_s, 4), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1000 / args.steps, 4),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
        "dtype": "f16 activations, u4 weights, f32 accumulate", "data": "synthetic (seeded)",
        "config": stack_config(args, world),
        "GBps": round(nbytes * args.steps / dt / 1e9, 3),
        "cpu_baseline": {"value": round(tok_s, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(tok_s, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "MLX (the reference's arithmetic) is not installable here; this is the oracle restatement",
    }
    print(json.dumps(out), flush=True)


def run_case(args):
    """One kernel on one shape; prints one JSON line.  Used for ncu captures.

    M,N,K          quantized matmul, 4 rotating weight copies (> L2 for the
                   BASELINE shapes)
    swiglu:M,I,K   fused SwiGLU gate/up, I rows each (4 rotating copies)
    b8:M,N,K       quantized matmul of 8-bit codes (groups of 64)
    topk:M,N,k     top-k of M rows of N fp16 logits"""
    import torch
    import qw_b200 as qw
    kind, _, spec = args.case.rpartition(":")
    dev = torch.device("cuda", 0)
    if kind == "topk":
        M, N, k = (int(v) for v in spec.split(","))
        lg = (torch.randn(M, N, device=dev) * 3).half()
        us = graph_time_us(torch, lambda: qw.topk(lg, k), dev, iters=max(3, args.steps))
        print(json.dumps({"case": ["topk", M, N, k], "us": round(us, 3),
                          "GBps_logits_read": round(2.0 * M * N / (us * 1e-6) / 1e9, 1)}), flush=True)
        return
    M, N, K = (int(v) for v in spec.split(","))
    if kind == "swiglu":
        us, gbs = kernel_microbench(torch, qw, M, 2 * N, K, dev, copies=4, iters=args.steps, swiglu=True)
        N = 2 * N
    else:
        us, gbs = kernel_microbench(torch, qw, M, N, K, dev, copies=4, iters=args.steps,
                                    bits=8 if kind == "b8" else 4)
    hbm_peak, _, src = peaks()
    print(json.dumps({"case": [M, N, K], "us": round(us, 3), "GBps": round(gbs, 1),
                      "frac_hbm": round(gbs / hbm_peak, 4), "peak_source": src,
                      "TFLOPs": round(2.0 * M * N * K / (us * 1e-6) / 1e12, 2)}), flush=True)


def run_tp_calls(args):
    """Per-call device time of the tensor-parallel row-parallel patterns on
    this world's shards (torchrun, N > 1): the o and down shards as a matmul
    alone, as a matmul into fp32 plus qw_allreduce_sum, and fused
    (qw_allreduce_matmul); the q|k|v and lm_head shards as matmuls.  Each
    pattern is a CUDA graph over 8 weight copies (more than L2 for the
    row-parallel shards), replayed 20 times after a barrier; max over ranks.
    Rank 0 prints one JSON line."""
    import torch
    import torch.distributed as dist
    import qw_b200 as qw
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    ar = tp.PeerAllreduce(2048 * synth.HIDDEN)
    copies, iters = 8, 20
    s = torch.cuda.Stream(dev)

    def timed(calls):
        with torch.cuda.stream(s):
            for _ in range(2):
                for f in calls:
                    f()
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for f in calls:
                f()
        with torch.cuda.stream(s):
            g.replay()
        s.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            for _ in range(iters):
                g.replay()
            e1.record(s)
        s.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) * 1000.0 / (iters * len(calls))], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        del g
        return round(t.item(), 2)

    out = {"metric": "per-call device time of TP shards (us, max over ranks)", "n_gpus": world, "M": 1}
    lins = {l.name: l for l in synth.layer_linears()}
    for name in ("o", "down"):
        N, K = tp.shard_shape(lins[name], world)
        sets = [make_weights(torch, qw, N, K, seed=100 * i + rank, dev=dev) for i in range(copies)]
        x = torch.randn(1, K, device=dev).half()
        y = torch.empty(1, N, dtype=torch.float16, device=dev)
        part = torch.empty(1, N, dtype=torch.float32, device=dev)

        def mm(w):
            return lambda: qw.quantized_matmul(x, *w, out=y)

        def two(w):
            return lambda: (qw.quantized_matmul(x, *w, out=part), ar(part, y))

        def fused(w):
            return lambda: ar.matmul(x, w, y)

        out[f"{name}_{N}x{K}"] = {"matmul": timed([mm(w) for w in sets]),
                                  "matmul_then_allreduce": timed([two(w) for w in sets]),
                                  "fused": timed([fused(w) for w in sets])}
        del sets
    for name, lin in (("qkv", lins["qkv"]), ("lm_head", synth.LM_HEAD)):
        N, K = tp.shard_shape(lin, world)
        sets = [make_weights(torch, qw, N, K, seed=100 * i + rank, dev=dev) for i in range(4 if name == "lm_head" else copies)]
        x = torch.randn(1, K, device=dev).half()
        y = torch.empty(1, N, dtype=torch.float16, device=dev)
        out[f"{name}_{N}x{K}"] = {"matmul": timed([(lambda w=w: qw.quantized_matmul(x, *w, out=y)) for w in sets])}
        del sets
    out["device_status"] = qw.device_status(local, clear=False)
    dist.barrier()
    ar.close()
    dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=synth.LAYERS)
    ap.add_argument("--skip-extra", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--tp-allreduce", choices=["peer", "nccl"], default="peer",
                    help="exchange of the row-parallel partial sums under torchrun")
    ap.add_argument("--case", default=None,
                    help="M,N,K | swiglu:M,I,K | b8:M,N,K | topk:M,N,k: time one kernel on one shape only "
                         "(small device footprint, for ncu)")
    ap.add_argument("--tp-calls", action="store_true",
                    help="under torchrun: per-call times of the tensor-parallel shards and exchanges")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.tp_calls:
        run_tp_calls(args)
    elif args.case:
        run_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
