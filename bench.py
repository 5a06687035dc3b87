"""Benchmark of the int4 group-32 weight-only matmul path on B200 (one JSON line on rank 0).

Default workload: the Qwen2.5-32B dense decode stack, 64 layers of
random int4 group-32 weights (hidden 5120, intermediate 27648, 40 query / 8 KV heads x 128),
tensor-parallel over the ranks: q/k/v and gate/up column-parallel, o and down row-parallel with
an all-reduce after each (a peer-memory kernel fused with the row-parallel GEMV, or NCCL). M = 1
token per step by default (--rows 8 for the batched decode); the activations between the
projections stay fp32. One step = one decode pass over the 64 layers' projections from a CUDA
graph; 17.6 GB of weights per step at TP 1 (> L2, no flush needed).

Metric: decode tokens/s (strong scaling: the same model over N GPUs). Also in the line: the
dominant kernel (the gate/up GEMV + SwiGLU) timed alone against the measured HBM bandwidth, the
reference's CPU path timed on the host cores, the step through pinned host copies (e2e), a
parity check of one layer against the oracle, and at N = 1 the Qwen3-8B decode projections
(configs[1]) in GB/s.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config qwen2.5-32b|qwen3-8b|gemv|prefill|moe|attn] [--rows M]

Other configs: qwen3-8b (configs[1], GB/s; at --gpus N independent replicas), gemv,
prefill (configs[2], TFLOP/s), moe (configs[3], tokens/s; expert-parallel at N > 1), attn (the
decode attention row). --gpus N > 1 runs under torchrun, one rank per GPU; time = max over ranks
of the device-timed region. --impl reference times the reference's CPU dequantise-then-matmul
path (restated in oracle/) on this host's cores, on a bounded sample of the same workload.
"""
import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HIDDEN, INTER, LAYERS = 4096, 12288, 36
QKV_N = 4096 + 2 * 1024


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


# ------------------------------------------------------------------ workloads
def qwen3_8b_matrices():
    """(name, N, K, gateup) of one layer, in execution order."""
    return [("qkv", QKV_N, HIDDEN, False), ("gate_up", 2 * INTER, HIDDEN, True), ("down", HIDDEN, INTER, False)]


def int4_param_bytes(N, K):
    return N * K // 2 + N * (K // 32) * 2


def gen_int4_cuda(N, K, gen, gain=None, k_full=None):
    """Random int4 weights [N, K] (two's-complement codes packed along K, fp16 group scales).
    gain None: codes uniform in -8..7, scales |N(0, 0.02)| + 1e-4. gain g: a model-like matrix
    whose y = W x (summed over k_full inputs, K of them on this rank) has rms g * rms(x): codes
    uniform in -7..7 (zero mean, as quantised weights are; E[v^2] = 280/15), scales
    sigma * (|z| + 0.005) with E[(|z| + 0.005)^2] = 1.008. Zero-mean codes matter: with codes of
    mean -0.5 and positive scales every output shares a common offset that the next projection's
    32-groups add coherently."""
    if gain is None:
        qk = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=gen)
        s = ((torch.randn(N, K // 32, device="cuda", generator=gen) * 0.02).abs() + 1e-4).to(torch.float16)
        return qk, s
    u = torch.randint(0, 15, (N, K), dtype=torch.uint8, device="cuda", generator=gen)
    nib = u + (u >= 8).to(torch.uint8)                 # nibbles 0..7, 9..15: v = -7..7, never -8
    qk = nib[:, 0::2] | (nib[:, 1::2] << 4)
    del u, nib
    sigma = gain / math.sqrt(280.0 / 15.0 * (k_full or K) * 1.008)
    s = ((torch.randn(N, K // 32, device="cuda", generator=gen).abs() + 0.005) * sigma).to(torch.float16)
    return qk.contiguous(), s


class DecodeStack:
    """The Qwen3-8B projection stack on one GPU (libonpu dense matrices). mode "chain": the whole
    step is one GEMV chain (onpu_chain_*), every link ordered after its predecessor as in a real
    decode step; mode "launches": one onpu_dense_mv_dev launch per matrix."""

    def __init__(self, M, seed, layers=LAYERS, mode="launches", act="f32"):
        from opennpu_b200 import dense
        self.dense = dense
        # act: the MLP activation between gate/up and down. "f32": the SwiGLU epilogue writes fp32
        # and the down GEMV stages it as two fp16 halves per value (the reference's fp32 chain,
        # reference.py:55-57, :84); "bf16": rounded once to bf16 (the reference's NPU input rounding)
        self.act = "bf16" if mode == "chain" else act
        self.M, self.mode = M, mode
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed)
        self.layers = []
        for _ in range(layers):
            mats = {}
            for name, N, K, gu in qwen3_8b_matrices():
                qk, s = gen_int4_cuda(N, K, gen)
                mats[name] = dense.DenseMatrix.from_int4(qk, s, gateup=gu)
                del qk, s
            self.layers.append(mats)
        torch.cuda.synchronize()
        if M > self.layers[0]["down"].max_f32_rows():
            self.act = "bf16"                 # the fp32 rows would not fit in shared memory
        self.x_all = torch.randn(layers, M, HIDDEN, device="cuda", generator=gen).to(torch.bfloat16)
        self.x = [self.x_all[l] for l in range(layers)]
        self.y_qkv = torch.empty(M, QKV_N, device="cuda")
        self.a = torch.empty(M, INTER, device="cuda", dtype=torch.float32 if self.act == "f32" else torch.bfloat16)
        self.epi_gu = dense.EPI_SWIGLU_F32 if self.act == "f32" else dense.EPI_SWIGLU
        self.y = torch.empty(M, HIDDEN, device="cuda")
        per_layer = 0
        for name, N, K, gu in qwen3_8b_matrices():
            per_layer += int4_param_bytes(N, K) + M * K * 2
        per_layer += M * QKV_N * 4 + M * INTER * self.a.element_size() + M * HIDDEN * 4
        per_layer += M * INTER * (self.a.element_size() - 2)          # down reads the activation
        self.bytes_per_step = per_layer * layers
        self.weight_bytes_per_step = sum(int4_param_bytes(N, K) for _, N, K, _ in qwen3_8b_matrices()) * layers
        self.chain = None
        if mode == "chain":
            self.chain = dense.DenseChain()
            prev = -1
            for l, mats in enumerate(self.layers):
                prev = self.chain.add(mats["qkv"], self.x[l], self.y_qkv, dep=prev)
                prev = self.chain.add(mats["gate_up"], self.x[l], self.a, epi=dense.EPI_SWIGLU, dep=prev)
                prev = self.chain.add(mats["down"], self.a, self.y, dep=prev)
            self.chain.prepare()
        self.launches_per_step = 1 if mode == "chain" else 3 * layers

    def dominant(self):
        """The dominant kernel of the step alone: (callable, algorithmic bytes per launch,
        launches per call, kernel name). Chain mode: the chain kernel is the step's only launch;
        launches mode: gate_up GEMV + SwiGLU epilogue over all layers."""
        d = self.dense
        if self.chain is not None:
            return self.chain.run, self.bytes_per_step, 1, "gemv_chain_kernel (one launch = the whole step)"
        N, K = 2 * INTER, HIDDEN
        nbytes = int4_param_bytes(N, K) + self.M * K * 2 + self.M * INTER * self.a.element_size()

        def run():
            for l, mats in enumerate(self.layers):
                mats["gate_up"].mv(self.x[l], out=self.a, epi=self.epi_gu)
        return run, nbytes, len(self.layers), "gemv_int4_kernel gate_up 24576x4096 + SwiGLU"

    def step(self):
        if self.chain is not None:
            self.chain.run()
            return
        for l, mats in enumerate(self.layers):
            mats["qkv"].mv(self.x[l], out=self.y_qkv)
            mats["gate_up"].mv(self.x[l], out=self.a, epi=self.epi_gu)
            mats["down"].mv(self.a, out=self.y)

    def step_e2e(self, hx, hy_qkv, hy):
        """One step through the public API with host buffers: pinned bf16 activations of every
        layer -> device, the step, the last layer's q/k/v and down outputs -> pinned host."""
        self.x_all.copy_(hx, non_blocking=True)
        self.step()
        hy_qkv.copy_(self.y_qkv, non_blocking=True)
        hy.copy_(self.y, non_blocking=True)
        torch.cuda.current_stream().synchronize()

    def step_host(self, xs_host, ys_host):
        """The same pass through the reference ABI's host-pointer call (onpu_dense_mv): fp32 host
        inputs/outputs, copies and a synchronisation inside every call, SwiGLU on the host."""
        from opennpu_b200 import libonpu as L
        lib = L.load()
        for l, mats in enumerate(self.layers):
            x = xs_host[l]
            lib.onpu_dense_mv(mats["qkv"].h, L.fp(x), self.M, L.fp(ys_host["qkv"]))
            lib.onpu_dense_mv(mats["gate_up"].h, L.fp(x), self.M, L.fp(ys_host["gate_up"]))
            h = ys_host["gate_up"]
            g, u = h[:, :INTER], h[:, INTER:]
            a = np.ascontiguousarray(g / (1.0 + np.exp(-g)) * u, np.float32)
            lib.onpu_dense_mv(mats["down"].h, L.fp(a), self.M, L.fp(ys_host["down"]))
        err = L.last_error()
        if err:
            raise RuntimeError(err)


# Qwen3-14B: prefill dequant-GEMMs
P_HIDDEN, P_INTER = 5120, 17408


class PrefillStack:
    """Qwen3-14B MLP projections for M prefill tokens on the tensor cores (gate_up with
    the SwiGLU epilogue, then down), `layers` layers of synthetic int4 weights."""

    def __init__(self, M, seed, layers=2, rank=0, world=1, group=None):
        """world > 1: tensor parallelism (tp.TPMLP): this rank's gate/up rows (column-parallel)
        and down K block (row-parallel, NCCL all-reduce of the [M, hidden] output); every rank
        generates only its own shards."""
        from opennpu_b200 import dense, tp
        self.dense = dense
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed)
        self.layers = []
        ir = P_INTER // world
        for _ in range(layers):
            gu = gen_int4_cuda(2 * ir, P_HIDDEN, gen)
            dn = gen_int4_cuda(P_HIDDEN, ir, gen)
            self.layers.append(tp.TPMLP(gu, dn, group=group))
            del gu, dn
        torch.cuda.synchronize()
        self.M, self.world = M, world
        self.x = torch.randn(M, P_HIDDEN, device="cuda", generator=gen).to(torch.bfloat16)
        self.a = torch.empty(M, ir, device="cuda", dtype=torch.bfloat16)
        self.y = torch.empty(M, P_HIDDEN, device="cuda")
        # whole-model FLOPs (the same at every rank count: strong scaling)
        self.flops_gu = 2 * M * (2 * P_INTER) * P_HIDDEN
        self.flops_per_step = layers * (self.flops_gu + 2 * M * P_HIDDEN * P_INTER)
        self.flops_gu_rank = self.flops_gu // world
        self.launches_per_step = 4 * layers            # activation copy + GEMM, per matrix

    def step(self):
        for mlp in self.layers:
            mlp(self.x, self.a, self.y)

    def dominant(self):
        d = self.dense

        def run():
            for mlp in self.layers:
                mlp.gu.mm(self.x, self.a, epi=d.EPI_SWIGLU)
        return run, self.flops_gu_rank, len(self.layers)


_CPU_CACHE = {}


def _cpu_cached(key, make):
    """CPU sample weights, generated once per process (the reference arm times many steps)."""
    if key not in _CPU_CACHE:
        _CPU_CACHE[key] = make()
    return _CPU_CACHE[key]


def cpu_prefill_sample(M_cpu=128, seconds=10.0, seed=0):
    """The reference's CPU path on the prefill shapes: dequantise per 32 (w = v * s) then fp32
    matmul with all host threads, on M_cpu tokens; TFLOP/s."""
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)

    def make():
        mats = []
        for N, K in ((2 * P_INTER, P_HIDDEN), (P_HIDDEN, P_INTER)):
            v = torch.randint(-8, 8, (N, K), generator=g, dtype=torch.int8)
            sc = (torch.randn(N, K // 32, generator=g).abs() * 0.02 + 1e-4).half()
            mats.append((v, sc))
        return mats
    mats = _cpu_cached(("prefill", seed), make)
    x = torch.randn(M_cpu, P_HIDDEN, generator=g).bfloat16().float()
    flops, t0, n = 0, time.perf_counter(), 0
    while True:
        h = x
        for (v, sc), act in zip(mats, (True, False)):
            w = (v.float().view(v.shape[0], -1, 32) * sc.float().unsqueeze(-1)).view(v.shape[0], -1)
            h = h @ w.T
            flops += 2 * h.shape[0] * w.shape[0] * w.shape[1]
            if act:
                gte, up = h[:, :P_INTER], h[:, P_INTER:]
                h = gte * torch.sigmoid(gte) * up
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return flops / dt / 1e12, torch.get_num_threads(), f"{n} x one Qwen3-14B MLP (gate_up + SwiGLU + down, dequant + fp32 matmul) on {M_cpu} tokens"


def run_prefill(args):
    rank, world, local = dist_setup(args.gpus)
    _, tflops_peak, peak_kind = peaks()
    M = args.m if args.m > 1 else 2048
    group = torch.distributed.group.WORLD if world > 1 else None
    work = PrefillStack(M, seed=2000 + rank, layers=2, rank=rank, world=world, group=group)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(max(args.warmup, 1)):
            work.step()
    s.synchronize()
    from opennpu_b200 import dense
    dense.check_device()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        work.step()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            graph.replay()
    s.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    with torch.cuda.stream(s):
        for _ in range(args.steps):
            graph.replay()
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    dense.check_device()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    tflops = work.flops_per_step / (ms_step * 1e-3) / 1e12          # the whole model, over all ranks

    run_dom, dom_flops, dom_n = work.dominant()
    gdom = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gdom, stream=s):
        run_dom()
    with torch.cuda.stream(s):
        for _ in range(3):
            gdom.replay()
    reps = 20
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(s)
    with torch.cuda.stream(s):
        for _ in range(reps):
            gdom.replay()
    d1.record(s)
    d1.synchronize()
    dom_us = d0.elapsed_time(d1) * 1e3 / (reps * dom_n)
    del gdom

    e2e = None
    if not args.no_e2e:
        hx = torch.empty(work.x.shape, dtype=torch.bfloat16, pin_memory=True)
        hx.copy_(work.x)
        hy = torch.empty(work.y.shape, dtype=torch.float32, pin_memory=True)
        with torch.cuda.stream(s):
            for i in range(3 + 10):
                if i == 3:
                    t0 = time.perf_counter()
                work.x.copy_(hx, non_blocking=True)
                work.step()
                hy.copy_(work.y, non_blocking=True)
                s.synchronize()
        dt = (time.perf_counter() - t0) / 10
        e2e = {"value": round(work.flops_per_step / dt / 1e12, 2), "unit": "TFLOP/s",
               "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": hy.numel() * 4,
               "ms_per_step": round(dt * 1e3, 3),
               "path": "onpu_dense_mm_dev with pinned host input/output copies and a host synchronisation per step"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, sample = cpu_prefill_sample(seconds=args.cpu_seconds)
        cpu = {"value": round(v, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        achieved = dom_flops / (dom_us * 1e-6) / 1e12
        line = {
            "metric": "int4 prefill dequant-GEMM TFLOP/s (Qwen3-14B MLP, tcgen05)", "value": round(tflops, 2),
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 weights dequantised to fp16, fp16 x fp16 -> fp32",
            "data": "synthetic (seeded random int4 weights, fp16 scales, bf16 N(0,1))",
            "config": {"workload": "qwen3-14b-prefill-mlp", "M": M, "layers": len(work.layers),
                       "matrices": "gate_up 34816x5120 + SwiGLU, down 5120x17408",
                       "parallelism": f"tp{world}", "l2": "weights larger than L2 (no flush needed)",
                       "collective": "NCCL all-reduce of the [M, 5120] fp32 output after down" if world > 1 else None,
                       "cuda_graph": True},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 1), "peak": tflops_peak, "unit": "TFLOP/s",
                         "frac": round(achieved / tflops_peak, 4), "peak_kind": peak_kind + " (bf16 dense, burst)",
                         "traffic": None, "kernel": "dqgemm_kernel gate_up 34816x5120 + SwiGLU",
                         "flops_per_launch": dom_flops, "us_per_launch": round(dom_us, 3)},
            "cpu_baseline": cpu, "e2e": e2e, "clocks": clk, "gpu_launches": work.launches_per_step * args.steps,
        }
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        torch.distributed.destroy_process_group()


M_E, M_K, M_HIDDEN, M_INTER, M_LAYERS = 128, 8, 2048, 768, 48

# ------------------------------------------------------------------ decode attention
A_HQ, A_HKV, A_D, A_LAYERS = 32, 8, 128, 36          # Qwen3-8B


def attn_step_bytes(S, layers=A_LAYERS):
    return 2 * A_HKV * S * A_D * 2 * layers               # every layer's bf16 K and V read once


def cpu_attn_sample(S, seconds=10.0, seed=0):
    """The reference's own onpu_attn_step_bf16 (onpu_cpu.cpp:173-229, compiled into oracle/_ref;
    its thread pool uses every host core) on one layer's cache of the same shape, repeated for
    about `seconds`. Falls back to the oracle's numpy restatement when oracle/_ref is absent.
    Returns (GB/s of cache read, cores, kind, sample)."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    q = rng.normal(size=(A_HQ, A_D)).astype(np.float32)
    K = O.f32_to_bf16_bits(rng.normal(size=(A_HKV, S, A_D)).astype(np.float32))
    V = O.f32_to_bf16_bits(rng.normal(size=(A_HKV, S, A_D)).astype(np.float32))
    L = O.ref_lib()
    if L is not None:
        run, kind = (lambda: O.attn_step_ref(L, q, K, V, bf16=True)), "reference"
    else:
        Kf, Vf = O.bf16_bits_to_f32(K), O.bf16_bits_to_f32(V)
        run, kind = (lambda: O.attn_step(q, Kf, Vf)), "port"
    run()
    n, t0 = 0, time.perf_counter()
    while True:
        run()
        n += 1
        dt = time.perf_counter() - t0
        if dt >= seconds:
            break
    gbs = attn_step_bytes(S, 1) * n / dt / 1e9
    sample = f"{n} x one Qwen3-8B layer's decode attention (Hq 32, Hkv 8, D 128, S {S}, bf16 cache)"
    return gbs, os.cpu_count(), kind, sample


def run_attn(args):
    """Config attn: one decode token's attention over all 36 layers of Qwen3-8B at `--context`
    tokens (bf16 KV caches, 604 MB at 4k: larger than L2), through onpu_attn_step_dev, the step's
    36 calls captured in a CUDA graph as the other configs' steps are."""
    from opennpu_b200 import libonpu as L
    from opennpu_b200.attn import attn_step
    rank, world, local = dist_setup(args.gpus)
    hbm_peak, _, peak_kind = peaks()
    S = args.context
    g = torch.Generator(device="cuda").manual_seed(3000 + rank)
    q = torch.randn(A_HQ, A_D, device="cuda", generator=g)
    ks = [torch.randn(A_HKV, S, A_D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(A_LAYERS)]
    vs = [torch.randn(A_HKV, S, A_D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(A_LAYERS)]
    out = torch.empty(A_HQ, A_D, device="cuda")
    s = torch.cuda.Stream()

    def step():
        for k, v in zip(ks, vs):
            attn_step(q, k, v, out=out, stream=s)

    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            step()
    s.synchronize()
    assert L.load().onpu_check_device() == 0, L.last_error()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        step()
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            graph.replay()
    s.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    with torch.cuda.stream(s):
        for _ in range(args.steps):
            graph.replay()
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    assert L.load().onpu_check_device() == 0, L.last_error()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    nbytes = attn_step_bytes(S)
    gbs = nbytes * world / (ms_step * 1e-3) / 1e9
    us_call = ms_step * 1e3 / A_LAYERS

    e2e = None
    if not args.no_e2e:
        # the reference ABI: host q, host caches (copied up by the library each call), host out
        lib = L.load()
        hk = [k.cpu().view(torch.int16).numpy() for k in ks[:4]]
        hv = [v.cpu().view(torch.int16).numpy() for v in vs[:4]]
        hq = q.cpu().numpy()
        ho = np.empty((A_HQ, A_D), np.float32)
        fp = lambda a: a.ctypes.data_as(L.F)
        n_e2e, t0 = 0, None
        for i in range(2 + 3):
            if i == 2:
                t0 = time.perf_counter()
            for l in range(A_LAYERS):
                lib.onpu_attn_step_bf16(fp(hq), A_HQ, A_D, fp(hk[l % 4]), fp(hv[l % 4]), A_HKV, S, S * A_D, A_D,
                                        None, None, A_D ** -0.5, fp(ho))
            n_e2e += i >= 2
        assert L.last_error() is None, L.last_error()
        dt = (time.perf_counter() - t0) / n_e2e
        e2e = {"value": round(nbytes / dt / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": A_LAYERS * (2 * A_HKV * S * A_D * 2 + A_HQ * A_D * 4),
               "d2h_bytes_per_step": A_LAYERS * A_HQ * A_D * 4, "ms_per_step": round(dt * 1e3, 3),
               "path": "onpu_attn_step_bf16 (the reference ABI: host q, host caches copied up each call, "
                       "host out), 36 calls per step"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, kind, sample = cpu_attn_sample(S, seconds=args.cpu_seconds)
        cpu = {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": kind, "sample": sample}
    if rank == 0:
        achieved = attn_step_bytes(S, 1) / (us_call * 1e-6) / 1e9
        traffic = json.loads((ROOT / "profiles" / "traffic.json").read_text()).get(f"attn/{S}")
        line = {
            "metric": "decode attention KV-cache GB/s (Qwen3-8B, 36 layers, bf16 cache)", "value": round(gbs, 2),
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 cache, fp32 arithmetic (q and P as three bf16 parts on the tensor cores)",
            "data": "synthetic (seeded N(0,1) q and caches)",
            "config": {"workload": "qwen3-8b-decode-attention", "context": S, "layers": A_LAYERS,
                       "heads": f"{A_HQ} query / {A_HKV} kv, D {A_D}", "parallelism": f"replicas{world}",
                       "l2": "36 distinct caches, larger than L2 (no flush needed)", "cuda_graph": True},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind, "traffic": traffic,
                         "kernel": "attn_split_tc_kernel<128> + attn_combine_kernel (one call, one layer)",
                         "algorithmic_bytes_per_launch": attn_step_bytes(S, 1), "us_per_launch": round(us_call, 3)},
            "cpu_baseline": cpu, "e2e": e2e, "clocks": clk, "gpu_launches": 2 * A_LAYERS * args.steps,
        }
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        torch.distributed.destroy_process_group()


def moe_expert_bytes():
    """int4 codes + fp16 scales of one expert's gate_up (1536x2048) and down (2048x768)."""
    return int4_param_bytes(2 * M_INTER, M_HIDDEN), int4_param_bytes(M_HIDDEN, M_INTER)


class MoEStack:
    """Qwen3-30B-A3B MoE layers (router 128 experts top-8 renormalised, experts
    gate_up 1536x2048 + SwiGLU and down 2048x768 in int4), T tokens. One step = the router and the
    routed-expert FFN of every layer; each layer has its own weights and its own bf16 N(0,1)
    input rows, so the routing (and the experts read) differs per layer."""

    def __init__(self, T, seed, layers=M_LAYERS, rank=0, world=1, group=None, ep="gather"):
        """world > 1: expert parallelism, this rank holds experts [rank * E / world, ...) of every
        layer and its own T tokens (moe.EPMoELayer: all-gather of tokens and routing, reduce-scatter
        of the outputs). Router weights are the same on every rank."""
        from opennpu_b200 import moe
        self.moe = moe
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed + 7919 * rank)
        rgen = torch.Generator(device="cuda")
        rgen.manual_seed(seed)
        el = M_E // world
        self.T, self.layers, self.world, self.rank = T, [], world, rank
        for _ in range(layers):
            wr = (torch.randn(M_E, M_HIDDEN, device="cuda", generator=rgen) * 0.02).to(torch.bfloat16)
            gq = torch.randint(0, 256, (el, 2 * M_INTER, M_HIDDEN // 2), dtype=torch.uint8, device="cuda",
                               generator=gen)
            gs = ((torch.randn(el, 2 * M_INTER, M_HIDDEN // 32, device="cuda", generator=gen) * 0.02).abs()
                  + 1e-4).half()
            dq = torch.randint(0, 256, (el, M_HIDDEN, M_INTER // 2), dtype=torch.uint8, device="cuda", generator=gen)
            ds = ((torch.randn(el, M_HIDDEN, M_INTER // 32, device="cuda", generator=gen) * 0.02).abs()
                  + 1e-4).half()
            ffn = moe.ExpertFFN(gq, gs, dq, ds)
            del gq, gs, dq, ds
            kind = moe.EPMoELayerA2A if ep == "a2a" else moe.EPMoELayer
            ep_layer = kind(wr, ffn, rank, world, M_E, group=group, k=M_K) if world > 1 else None
            self.layers.append((wr, ffn, ep_layer))
        torch.cuda.synchronize()
        self.x = torch.randn(layers, T, M_HIDDEN, device="cuda", generator=gen).to(torch.bfloat16)
        self.ids = torch.empty(layers, T, M_K, dtype=torch.int32, device="cuda")
        self.w = torch.empty(layers, T, M_K, device="cuda")
        self.y = torch.empty(layers, T, M_HIDDEN, device="cuda")
        self.ep = ep
        self.bufs = ([e.buffers(T, M_HIDDEN) for _, _, e in self.layers] if world > 1 and ep == "gather"
                     else None)
        # router (+ job lists), gate_up, down, combine; with expert parallelism the job builder runs
        # separately (the ids are all-gathered first)
        self.launches_per_step = (4 if world == 1 else 5) * layers
        self.lib = __import__("opennpu_b200.libonpu", fromlist=["load"]).load()

    def step(self, stream):
        sp = stream.cuda_stream
        for l, (wr, ffn, ep) in enumerate(self.layers):
            x = self.x[l]
            if ep is not None:
                if self.ep == "a2a":
                    self.y[l].copy_(ep(x, stream=stream))
                else:
                    self.y[l].copy_(ep(x, self.bufs[l], stream=stream))
                continue
            ffn.layer(x, wr, M_K, out=self.y[l], ids=self.ids[l], w=self.w[l], stream=stream)

    def algorithmic_bytes(self):
        """Per step and GPU: every layer's router weights and input rows, the int4 bytes of this
        GPU's experts that the (all ranks') tokens selected, each read once, the ids/weights and the
        fp32 outputs."""
        gu, dn = moe_expert_bytes()
        b = 0
        el = M_E // self.world
        for l in range(len(self.layers)):
            if self.world > 1:
                if self.ep == "a2a":          # the all-to-all form keeps no gathered ids: route and gather here
                    from opennpu_b200 import moe
                    mine, _ = moe.route(self.x[l], self.layers[l][0], M_K)
                    every = torch.empty(self.world * self.T, M_K, dtype=mine.dtype, device=mine.device)
                    torch.distributed.all_gather_into_tensor(every, mine.contiguous())
                    ids = every.cpu().numpy()
                else:
                    ids = self.bufs[l]["ids_all"].cpu().numpy()
                nexp = len({int(e) for e in np.unique(ids) if self.rank * el <= e < (self.rank + 1) * el})
                toks = self.T * self.world
            else:
                nexp = len(np.unique(self.ids[l].cpu().numpy()))
                toks = self.T
            b += nexp * (gu + dn) + M_E * M_HIDDEN * 2 + toks * M_HIDDEN * (2 + 4) + toks * M_K * 8
        return b


def cpu_moe_sample(T, seconds=10.0, seed=0):
    """The reference's CPU MoE layer (opennpu/native/reference.py:71-84): router softmax / top-8 /
    renormalise, then per selected expert dequantise (v * s) and fp32 matmuls with SwiGLU, all host
    threads; layer tokens/s."""
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)

    def make():
        wr = (torch.randn(M_E, M_HIDDEN, generator=g) * 0.02).bfloat16().float()
        gv = torch.randint(-8, 8, (M_E, 2 * M_INTER, M_HIDDEN), dtype=torch.int8, generator=g)
        gsc = (torch.randn(M_E, 2 * M_INTER, M_HIDDEN // 32, generator=g).abs() * 0.02 + 1e-4).half()
        dv = torch.randint(-8, 8, (M_E, M_HIDDEN, M_INTER), dtype=torch.int8, generator=g)
        dsc = (torch.randn(M_E, M_HIDDEN, M_INTER // 32, generator=g).abs() * 0.02 + 1e-4).half()
        return wr, gv, gsc, dv, dsc
    wr, gv, gsc, dv, dsc = _cpu_cached(("moe", seed), make)

    def deq(v, s):
        N, K = v.shape
        return (v.view(N, K // 32, 32).float() * s.float()[..., None]).view(N, K)

    def layer(x):
        prob = (x @ wr.T).softmax(-1)
        w, sel = prob.topk(M_K, -1)
        w = w / w.sum(-1, keepdim=True)
        out = torch.zeros_like(x)
        for e in sel.unique().tolist():
            rows = (sel == e).any(-1).nonzero().flatten()
            we = (w * (sel == e)).sum(-1)[rows, None]
            h = x[rows] @ deq(gv[e], gsc[e]).T
            a = torch.nn.functional.silu(h[:, :M_INTER]) * h[:, M_INTER:]
            out[rows] += we * (a @ deq(dv[e], dsc[e]).T)
        return out

    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 1:
        layer(torch.randn(T, M_HIDDEN, generator=g).bfloat16().float())
        n += 1
    dt = time.perf_counter() - t0
    return n * T / dt, torch.get_num_threads(), f"{n} x one Qwen3-30B-A3B MoE layer (router + dequant + fp32 experts) on {T} tokens"


def run_moe(args):
    rank, world, local = dist_setup(args.gpus)
    hbm, _, peak_kind = peaks()
    T = args.m if args.m > 0 else 1
    layers = args.layers
    group = torch.distributed.group.WORLD if world > 1 else None
    work = MoEStack(T, seed=3000, layers=layers, rank=rank, world=world, group=group, ep=args.ep)
    assert work.lib.onpu_moe_set_fused(args.moe_fused) >= 0
    fused = args.moe_fused == 1
    if fused and world == 1:
        work.launches_per_step = 2 * layers             # router (+ job lists), the persistent expert FFN
    elif fused:
        work.launches_per_step = 3 * layers             # router, job lists, the persistent expert FFN
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(max(args.warmup, 1)):
            work.step(s)
    s.synchronize()
    from opennpu_b200 import dense
    dense.check_device()
    # the all-to-all form reads its split sizes on the host: it runs eagerly, not from a graph
    graph = None
    if not (world > 1 and args.ep == "a2a"):
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            work.step(s)
        torch.cuda.synchronize()

    def replay():
        if graph is not None:
            graph.replay()
        else:
            work.step(s)
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            replay()
    s.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    with torch.cuda.stream(s):
        for _ in range(args.steps):
            replay()
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    dense.check_device()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    layer_us = ms_step * 1e3 / layers
    tok_s = T * world / (layer_us * 1e-6)
    nbytes = work.algorithmic_bytes()
    gbs = nbytes / (ms_step * 1e-3) / 1e9

    e2e = None
    if not args.no_e2e:
        hx = torch.empty(work.x.shape, dtype=torch.bfloat16, pin_memory=True)
        hx.copy_(work.x)
        hy = torch.empty(work.y.shape, dtype=torch.float32, pin_memory=True)
        with torch.cuda.stream(s):
            for i in range(3 + 10):
                if i == 3:
                    if world > 1:
                        torch.distributed.barrier()
                    t0 = time.perf_counter()
                work.x.copy_(hx, non_blocking=True)
                work.step(s)
                hy.copy_(work.y, non_blocking=True)
                s.synchronize()
        dt = (time.perf_counter() - t0) / 10
        if world > 1:
            t = torch.tensor([dt], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            dt = float(t.item())
        e2e = {"value": round(T * world / (dt / layers), 1), "unit": "tokens/s",
               "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": hy.numel() * 4,
               "ms_per_step": round(dt * 1e3, 3),
               "path": "onpu_moe_layer_dev per layer (EPMoELayer at N > 1; no graph), pinned host input/output "
                       "copies, a host synchronisation per step"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, sample = cpu_moe_sample(T, seconds=args.cpu_seconds)
        cpu = {"value": round(v, 2), "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        line = {
            "metric": "MoE layer tokens/s (Qwen3-30B-A3B: router + 128-expert top-8 int4 FFN)",
            "value": round(tok_s, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4 weights, bf16 inputs, fp32 activation between the projections, "
                                          "fp32 accumulate",
            "data": "synthetic (seeded random int4 experts, fp16 scales, bf16 N(0,1) tokens, N(0,0.02) router)",
            "config": {"workload": "qwen3-30b-a3b-moe-layer", "T": T, "T_per_gpu": T, "layers": layers,
                       "experts": M_E, "top_k": M_K, "hidden": M_HIDDEN, "expert_inter": M_INTER,
                       "parallelism": f"ep{world}" if world > 1 else "single", "us_per_layer": round(layer_us, 3),
                       "collective": (("NCCL all-to-all dispatch of routed token rows (+ counts) and combine"
                                       if args.ep == "a2a" else
                                       "NCCL all-gather (tokens, ids, weights) + reduce-scatter (outputs)")
                                      if world > 1 else None),
                       "l2": "selected experts of all layers per step exceed L2 (no flush needed)",
                       "cuda_graph": graph is not None,
                       "expert_ffn": "one persistent launch (gate_up + SwiGLU, down, combine)" if fused else
                                     "three launches (gate_up + SwiGLU GEMV, down GEMV, combine)"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(gbs / hbm, 4), "peak_kind": peak_kind + " (copy bandwidth)",
                         "traffic": None, "kernel": "whole MoE layer (router + job lists, then the expert FFN: "
                                                    + ("moe_ffn_kernel)" if fused else "gate_up + SwiGLU GEMV, down "
                                                       "GEMV, combine)"),
                         "bytes_per_step": nbytes},
            "cpu_baseline": cpu, "e2e": e2e, "clocks": clk, "gpu_launches": work.launches_per_step * args.steps,
        }
        print(json.dumps(line), flush=True)
    del graph
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


T_HIDDEN, T_INTER, T_QH, T_KVH, T_LAYERS = 5120, 27648, 40, 8, 64
# rms of N(0, 1) gate and up inputs for which silu(g) * u has rms 1 (E[(silu(c g) c u)^2] = 1)
SWIGLU_UNIT_GAIN = 1.269


def tp_layer0_parity(work, rank):
    """One layer of the timed stack against the oracle: layer 0's weights drawn again from the
    stack's seed, dequantised per 32 on the host and multiplied in float64 (reference.py:24-28,
    :55-57, :84 semantics; o takes q's output as the attention stand-in). At one rank with fp32
    activations between the projections the whole layer (all-reduced output) is checked; with
    more ranks, or with bf16 activations (rows that do not fit the fp32 staging), this rank's
    q/k/v shard: the reference's fp32 chain rounds nothing between the projections, and bf16
    roundings there are the engine's choice, not the kernel's arithmetic."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(work.seed)
    mats = [gen_int4_cuda(N, K, gen, gain=g, k_full=kf) for N, K, g, kf in work.gen_args]
    lay, M = work.layers[0], work.M
    x = torch.randn(M, T_HIDDEN, device="cuda", generator=torch.Generator(device="cuda").manual_seed(99))
    x = x.to(torch.bfloat16).to(work.x.dtype)
    b = lay.buffers(M)

    def mm(xx, qk, sc):                     # float64 x @ W.T, W dequantised a block of rows at a time
        qk, sc = qk.cpu(), sc.cpu().float()
        out = []
        for r0 in range(0, qk.shape[0], 2048):
            q = qk[r0:r0 + 2048]
            v = torch.stack([(q & 15).to(torch.int16), (q >> 4).to(torch.int16)], -1).view(q.shape[0], -1)
            v = torch.where(v >= 8, v - 16, v).double()
            w = (v.view(v.shape[0], -1, 32) * sc[r0:r0 + 2048].double()[..., None]).view(v.shape[0], -1)
            out.append(xx @ w.T)
        return torch.cat(out, 1)

    xd = x.double().cpu()
    if work.world == 1 and work.f32:
        y = lay(x, b).double().cpu()
        torch.cuda.synchronize()
        q = mm(xd, *mats[0])[:, :lay.nq]
        h = mm(q, *mats[1])
        gu = mm(h, *mats[2])
        I = gu.shape[1] // 2
        a = gu[:, :I] / (1 + torch.exp(-gu[:, :I])) * gu[:, I:]
        ref = mm(a, *mats[3])
        what = "layer 0 (q/k/v, o, gate/up + SwiGLU, down)"
    else:
        y = lay.qkv(x, b["qkv"], epi=work.tp.EPI_F32 if work.f32 else work.tp.EPI_BF16).double().cpu()
        torch.cuda.synchronize()
        ref = mm(xd, *mats[0])
        if not work.f32:
            ref = ref.float().bfloat16().double()
        what = f"layer 0, rank {rank}'s q/k/v shard"
    err = float((y - ref).norm() / ref.norm())
    mx = float((y - ref).abs().max())
    rms = float(ref.pow(2).mean().sqrt())
    return {"what": what, "rel_l2": err, "max_abs": mx, "ref_rms": rms,
            "ok": bool(err <= 1e-3 and mx <= 2e-2 * max(1.0, rms / 10.0)),
            "bound": "rel-L2 <= 1e-3; max-abs <= 2e-2 at a projection's output scale (rms 10), scaled by rms / 10"}


class TPStack:
    """Qwen2.5-32B decode projections, 64 layers of random int4 weights, tensor-parallel
    over the ranks: q/k/v and gate/up column-parallel (row blocks), o and down row-parallel (K
    blocks on 32-group boundaries) with an all-reduce of the fp32 partial outputs after each. Each
    rank generates only its own shards. Inside a layer each projection reads the previous one's
    output (o takes q's output as the stand-in for attention): fp32 for decode (M <= 8: every
    activation stays fp32, each GEMV stages it as two fp16 halves), else rounded to bf16. Layer
    l's q/k/v reads its own rms-1 input, the stand-in for the RMSNorm output a model feeds it
    (the norm is outside the matmul path; without it SwiGLU's quadratic response makes a chain of
    64 random layers grow or decay without bound); layer 0's input is the one the end-to-end
    timing copies from the host every step."""

    def __init__(self, M, rank, world, group, seed, layers=T_LAYERS, allreduce=None):
        from opennpu_b200 import tp
        self.tp = tp
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed)
        q, kv = T_QH * 128 // world, T_KVH * 128 // world
        i_r, h_r = T_INTER // world, T_HIDDEN // world
        self.layers = []
        # model-like scales keep every activation at rms ~1: each projection preserves rms, gate/up
        # outputs have rms 1.269 so that silu(g) * u has rms 1
        self.gen_args = [(q + 2 * kv, T_HIDDEN, 1.0, None), (T_HIDDEN, h_r, 1.0, T_HIDDEN),
                         (2 * i_r, T_HIDDEN, SWIGLU_UNIT_GAIN, None), (T_HIDDEN, i_r, 1.0, T_INTER)]
        for _ in range(layers):
            qkv, o, gu, dn = [gen_int4_cuda(N, K, gen, gain=g, k_full=kf) for N, K, g, kf in self.gen_args]
            self.layers.append(tp.TPDecoderLayer(qkv, o, gu, dn, q, group=group, allreduce=allreduce))
            del qkv, o, gu, dn
        torch.cuda.synchronize()
        self.M, self.world = M, world
        self.f32 = M <= min(lay.f32_rows for lay in self.layers)
        xin = torch.randn(layers, M, T_HIDDEN, device="cuda", generator=gen).to(torch.bfloat16)
        self.xin = xin.float() if self.f32 else xin          # each layer's q/k/v input
        self.x = self.xin[0]                                 # layer 0's: the host copies this one
        self.xs = [torch.empty(M, T_HIDDEN, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
        self.bufs = self.layers[0].buffers(M)
        shards = [(q + 2 * kv, T_HIDDEN), (T_HIDDEN, h_r), (2 * i_r, T_HIDDEN), (T_HIDDEN, i_r)]
        xb = 4 if self.f32 else 2
        self.bytes_per_layer = sum(int4_param_bytes(N, K) + M * K * xb + M * N * 4 for N, K in shards)
        # our kernels per layer: 4 GEMVs (o and down carry the peer all-reduce in the same launch)
        self.launches_per_step = 4 * layers
        self.seed, self.shapes = seed, shards

    def dominant(self, s):
        """The gate/up GEMV with its fused SwiGLU (the largest launch of the step) over every layer:
        (callable, algorithmic bytes per launch, launches per call, kernel name)."""
        tp, b = self.tp, self.bufs
        x, epi = (b["h"], tp.EPI_SWIGLU_F32) if self.f32 else (b["x2"], tp.EPI_SWIGLU)
        N, K = self.layers[0].gu.N, self.layers[0].gu.K
        nbytes = int4_param_bytes(N, K) + self.M * K * x.element_size() + self.M * (N // 2) * b["a"].element_size()

        def run():
            for lay in self.layers:
                lay.gu(x, b["a"], epi=epi, stream=s)
        return run, nbytes, len(self.layers), f"gemv_int4_kernel gate_up {N}x{K} + SwiGLU"

    def step(self):
        for i, lay in enumerate(self.layers):
            if self.f32:
                lay(self.xin[i], self.bufs)         # fp32 output y
            else:
                lay(self.xin[i], self.bufs, y_bf16=self.xs[i & 1])
        return self.bufs["y"]


def cpu_tp_sample(M, seconds=10.0, seed=0):
    """The reference's CPU path on one Qwen2.5-32B layer's projections (dequantise per 32 and fp32
    matmul, all host threads, M tokens); GB/s of int4 weights."""
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    from opennpu_b200 import tp

    def make():
        mats = []
        for name, N, K in tp.dense_layer_shapes(T_HIDDEN, T_INTER, T_QH, T_KVH):
            v = torch.randint(-8, 8, (N, K), dtype=torch.int8, generator=g)
            sc = ((torch.randn(N, K // 32, generator=g) * 0.02).abs() + 1e-4).to(torch.float16)
            mats.append((N, K, v, sc))
        return mats
    mats = _cpu_cached(("tp", seed), make)
    x = torch.randn(M, T_HIDDEN, generator=g).bfloat16().float()
    a = torch.randn(M, T_INTER, generator=g).bfloat16().float()
    layer_bytes = sum(int4_param_bytes(N, K) for N, K, _, _ in mats)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 1:
        for N, K, v, sc in mats:
            W = (v.view(N, K // 32, 32).float() * sc.float()[..., None]).view(N, K)
            (x if K == T_HIDDEN else (a if K == T_INTER else x)) @ W.T
        n += 1
    dt = time.perf_counter() - t0
    return n * layer_bytes / dt / 1e9, torch.get_num_threads(), f"{n} x one Qwen2.5-32B layer's 7 projections (dequant + fp32 matmul, M={M})"


def qwen3_8b_extra(args, hbm):
    """configs[1] at one GPU, kept beside the default line: the Qwen3-8B decode projections (36
    layers, M = 1, fp32 MLP activation) in GB/s and its gate/up launch against the HBM roofline."""
    work = DecodeStack(1, seed=1000, layers=LAYERS, act="f32")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(3):
            work.step()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        work.step()
    with torch.cuda.stream(s):
        for _ in range(3):
            g.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    steps = max(10, args.steps)
    e0.record(s)
    with torch.cuda.stream(s):
        for _ in range(steps):
            g.replay()
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / steps
    run_dom, dom_bytes, dom_n, dom_name = work.dominant()
    gd = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gd, stream=s):
        run_dom()
    with torch.cuda.stream(s):
        gd.replay()
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(s)
    with torch.cuda.stream(s):
        for _ in range(20):
            gd.replay()
    d1.record(s)
    d1.synchronize()
    us = d0.elapsed_time(d1) * 1e3 / (20 * dom_n)
    del g, gd
    gbs = work.bytes_per_step / (ms * 1e-3) / 1e9
    out = {"workload": "qwen3-8b-decode-projections (configs[1]), M = 1, 36 layers", "value": round(gbs, 2),
           "unit": "GB/s", "ms_per_step": round(ms, 4), "tokens_per_s": round(1e3 / ms, 1),
           "roofline": {"kernel": dom_name, "achieved": round(dom_bytes / (us * 1e-6) / 1e9, 1), "peak": hbm,
                        "frac": round(dom_bytes / (us * 1e-6) / 1e9 / hbm, 4), "us_per_launch": round(us, 3)}}
    del work
    torch.cuda.empty_cache()
    return out


def run_tp(args):
    rank, world, local = dist_setup(args.gpus)
    hbm, _, peak_kind = peaks()
    M = args.m
    layers = args.layers
    group = torch.distributed.group.WORLD if world > 1 else None
    allreduce = None
    if world > 1 and args.allreduce == "peer":
        from opennpu_b200.comm import PeerAllReduce
        # one communicator per call site (o, down): the fused GEMV's CTAs sum rows fixed by the shape
        allreduce = (PeerAllReduce(group, cap_floats=M * T_HIDDEN), PeerAllReduce(group, cap_floats=M * T_HIDDEN))
    work = TPStack(M, rank, world, group, seed=4000 + rank, layers=layers, allreduce=allreduce)
    f32 = work.f32
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(max(args.warmup, 1)):
            work.step()
    s.synchronize()
    from opennpu_b200 import dense
    dense.check_device()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        work.step()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            graph.replay()
    s.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    with torch.cuda.stream(s):
        for _ in range(args.steps):
            graph.replay()
    e1.record(s)
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    clk = clocks.stop()
    dense.check_device()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / args.steps
    tok_s = M / (ms_step * 1e-3)
    rank_bytes = work.bytes_per_layer * layers
    gbs_rank = rank_bytes / (ms_step * 1e-3) / 1e9

    # the dominant kernel alone: a graph of its launches over all layers, CUDA events on its stream
    run_dom, dom_bytes, dom_n, dom_name = work.dominant(s)
    gdom = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gdom, stream=s):
        run_dom()
    with torch.cuda.stream(s):
        for _ in range(3):
            gdom.replay()
    reps = 20
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(s)
    with torch.cuda.stream(s):
        for _ in range(reps):
            gdom.replay()
    d1.record(s)
    d1.synchronize()
    dom_us = d0.elapsed_time(d1) * 1e3 / (reps * dom_n)
    del gdom
    if world > 1:
        t = torch.tensor([dom_us], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        dom_us = float(t.item())

    e2e = None
    if not args.no_e2e:
        hx = torch.empty(work.x.shape, dtype=work.x.dtype, pin_memory=True)
        hx.copy_(work.x)
        hy = torch.empty(work.bufs["y"].shape, dtype=torch.float32, pin_memory=True)
        with torch.cuda.stream(s):
            for i in range(3 + 10):
                if i == 3:
                    if world > 1:
                        torch.distributed.barrier()
                    t0 = time.perf_counter()
                work.x.copy_(hx, non_blocking=True)
                graph.replay()
                hy.copy_(work.bufs["y"], non_blocking=True)
                s.synchronize()
        dt = (time.perf_counter() - t0) / 10
        if world > 1:
            t = torch.tensor([dt], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            dt = float(t.item())
        e2e = {"value": round(M / dt, 2), "unit": "tokens/s", "h2d_bytes_per_step": hx.numel() * hx.element_size(),
               "d2h_bytes_per_step": hy.numel() * 4, "ms_per_step": round(dt * 1e3, 3),
               "path": "TPDecoderLayer stack (onpu_dense_mv_f32_dev / onpu_dense_mv_dev; row-parallel o and down "
                       "fused with the peer all-reduce at N > 1) from a CUDA graph, pinned host input/output "
                       "copies and a host synchronisation per step (wall clock)"}
    del graph
    y_rms = float(work.bufs["y"].float().pow(2).mean().sqrt())      # the last layer's down output
    parity = tp_layer0_parity(work, rank)
    cpu = extra = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, sample = cpu_tp_sample(M, seconds=args.cpu_seconds)
        step_bytes = layers * sum(int4_param_bytes(N, K) for N, K in work.shapes)
        cpu = {"value": round(v * 1e9 / step_bytes * M, 4), "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": sample, "weight_gb_per_s": round(v, 3)}
    if rank == 0 and world == 1 and not args.no_extra:
        del work
        torch.cuda.empty_cache()
        extra = qwen3_8b_extra(args, hbm)
    if rank == 0:
        achieved = dom_bytes / (dom_us * 1e-6) / 1e9
        traffic = None
        tpf = ROOT / "profiles" / "traffic.json"
        if tpf.exists():
            traffic = json.loads(tpf.read_text()).get(f"qwen2.5-32b/tp{world}/M{M}")
        line = {
            "metric": "int4 dense decode stack tokens/s (Qwen2.5-32B, tensor-parallel)", "value": round(tok_s, 2),
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int4 weights, " + ("fp32 activations (two fp16 halves)" if f32 else "bf16 activations")
                     + ", fp32 accumulate",
            "data": "synthetic (seeded random zero-mean int4 weights, fp16 scales sized so every activation "
                    "stays at rms ~1; each layer's q/k/v input bf16 N(0,1), the stand-in for its RMSNorm output)",
            "config": tp_config(M, layers, world),
            "details": {"gb_per_s_all_ranks": round(gbs_rank * world, 1), "gb_per_s_per_gpu": round(gbs_rank, 1),
                        "bytes_per_step_per_gpu": rank_bytes, "l2": "inputs larger than L2 (no flush needed)",
                        "cuda_graph": True, "last_layer_output_rms": round(y_rms, 4),
                        "collective": (("the row-parallel GEMV fused with a one-shot all-reduce over NVLink peer "
                                        "memory (libonpu comm kernel)" if allreduce is not None else "NCCL all-reduce")
                                       + " (fp32) after o and down") if world > 1 else None},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_kind": peak_kind, "traffic": traffic,
                         "kernel": dom_name, "algorithmic_bytes_per_launch": dom_bytes,
                         "us_per_launch": round(dom_us, 3),
                         "step_gb_per_s_per_gpu": round(gbs_rank, 1), "step_frac": round(gbs_rank / hbm, 4)},
            "parity": parity, "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
            "gpu_launches": 4 * layers * args.steps,
        }
        if extra is not None:
            line["qwen3_8b_decode"] = extra
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        if allreduce is not None:
            for ar in allreduce:
                ar.close()
            torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def tp_config(M, layers, world):
    """The config dict of the qwen2.5-32b lines, the same in both arms."""
    return {"workload": "qwen2.5-32b-decode-projections-tp", "M": M, "layers": layers, "parallelism": f"tp{world}"}



class GemvRotation:
    """one 4096x4096 int4 GEMV, M=1; the step rotates over 32 weight copies (302 MB
    > L2) so every launch reads HBM."""

    def __init__(self, M, seed, copies=32, N=4096, K=4096):
        from opennpu_b200 import dense
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed)
        self.mats = []
        for _ in range(copies):
            qk, s = gen_int4_cuda(N, K, gen)
            self.mats.append(dense.DenseMatrix.from_int4(qk, s))
        self.M = M
        self.x = torch.randn(M, K, device="cuda", generator=gen).to(torch.bfloat16)
        self.y = torch.empty(M, N, device="cuda")
        self.bytes_per_step = copies * (int4_param_bytes(N, K) + M * K * 2 + M * N * 4)
        self.weight_bytes_per_step = copies * int4_param_bytes(N, K)
        self.launches_per_step = copies

    def dominant(self):
        nbytes = self.bytes_per_step // len(self.mats)
        return self.step, nbytes, len(self.mats), "gemv_int4_kernel 4096x4096"

    def step(self):
        for m in self.mats:
            m.mv(self.x, out=self.y)


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock, power and clock-event (throttle) reasons sampled every 10 ms through NVML while
    the timed region runs (short timed regions still get samples); nvidia-smi every 200 ms when
    NVML is not importable."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.nvml = None
        self.samples = []           # (sm MHz, reason bits)
        self.lines = []
        self.max_mhz = None
        self.stop_flag = threading.Event()

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            return
        except Exception:
            self.nvml = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 3.0:   # first sample before the timed region
                time.sleep(0.02)
            self.lines.clear()
        except OSError:
            self.proc = None

    def _poll(self):
        nv = self.nvml
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            nv.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self.stop_flag.is_set():
            try:
                self.samples.append((float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)),
                                     int(get_reasons(self.h))))
            except Exception:
                pass
            time.sleep(0.01)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml is not None:
            self.stop_flag.set()
            self.t.join(timeout=2)
            if not self.samples:
                return None
            reasons = sorted(n for n, bit in self.REASONS.items() if any(r & bit for _, r in self.samples))
            return {"sm_mhz": float(np.median([c for c, _ in self.samples])), "sm_max_mhz": self.max_mhz,
                    "reasons": reasons, "samples": len(self.samples), "source": "nvml, 10 ms"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [v.strip() for v in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "source": "nvidia-smi, 200 ms"}


# ------------------------------------------------------------------ CPU baseline (oracle port)
def cpu_reference_sample(M, seconds=10.0, seed=0):
    """The reference's CPU path on one Qwen3-8B layer's projections: dequantise per 32
    (reference.py:24-28 semantics, v * s) and fp32 matmul (reference.py:55-57), all host threads.
    Returns (GB/s with dequant per call, GB/s steady-state on pre-dequantised W, cores, sample)."""
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(seed)
    mats = []
    for name, N, K, gu in qwen3_8b_matrices():
        v = torch.randint(-8, 8, (N, K), dtype=torch.int8, generator=g)
        s = ((torch.randn(N, K // 32, generator=g) * 0.02).abs() + 1e-4).to(torch.float16)
        mats.append((N, K, v, s))
    x = torch.randn(M, HIDDEN, generator=g).to(torch.bfloat16).float()
    a = torch.randn(M, INTER, generator=g).to(torch.bfloat16).float()
    layer_bytes = sum(int4_param_bytes(N, K) for N, K, _, _ in mats)

    def deq(v, s):
        N, K = v.shape
        return (v.view(N, K // 32, 32).float() * s.float()[..., None]).view(N, K)

    def one_layer(pre=None):
        ys = []
        for i, (N, K, v, s) in enumerate(mats):
            W = pre[i] if pre is not None else deq(v, s)
            ys.append((x if K == HIDDEN else a) @ W.T)
        return ys

    one_layer()
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or n < 1:
        one_layer()
        n += 1
    dq = n * layer_bytes / (time.perf_counter() - t0) / 1e9
    pre = [deq(v, s) for _, _, v, s in mats]
    one_layer(pre)
    n2, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds / 2 or n2 < 1:
        one_layer(pre)
        n2 += 1
    ss = n2 * layer_bytes / (time.perf_counter() - t0) / 1e9
    sample = f"{n} x one Qwen3-8B layer's q/k/v, gate/up, down (dequant + fp32 matmul, M={M})"
    return dq, ss, torch.get_num_threads(), sample


# ------------------------------------------------------------------ runs
def dist_setup(n_gpus):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def run_ours(args):
    rank, world, local = dist_setup(args.gpus)
    hbm, _, peak_kind = peaks()
    M = args.m
    work = (DecodeStack(M, seed=1000 + rank, layers=args.layers, mode=args.mode, act=args.act)
            if args.config == "qwen3-8b"
            else GemvRotation(M, seed=1000 + rank))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for _ in range(max(args.warmup, 1)):
            work.step()
    s.synchronize()
    from opennpu_b200 import dense
    dense.check_device()

    use_graph = os.environ.get("ONPU_BENCH_GRAPH", "1") != "0"
    graph = None
    if use_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            work.step()
        torch.cuda.synchronize()

    def run_steps(k):
        with torch.cuda.stream(s):
            for _ in range(k):
                if graph is not None:
                    graph.replay()
                else:
                    work.step()

    run_steps(args.warmup)                              # warm-up of the timed path itself
    s.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(s)
    run_steps(args.steps)
    ev1.record(s)
    ev1.synchronize()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    dense.check_device()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
    ms_step = ms / args.steps
    gbs = work.bytes_per_step * world / (ms_step * 1e-3) / 1e9

    # roofline of the dominant kernel alone: a graph of its launches, CUDA events on its stream
    run_dom, dom_bytes, dom_n, dom_name = work.dominant()
    gdom = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gdom, stream=s):
        run_dom()
    with torch.cuda.stream(s):
        for _ in range(3):
            gdom.replay()
    reps = max(5, min(200, int(2000 / max(ms_step, 1e-3))))
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record(s)
    with torch.cuda.stream(s):
        for _ in range(reps):
            gdom.replay()
    d1.record(s)
    d1.synchronize()
    dom_us = d0.elapsed_time(d1) * 1e3 / (reps * dom_n)
    del gdom
    per_gpu_gbs = work.bytes_per_step / (ms_step * 1e-3) / 1e9

    # end to end through the public API with host buffers (pinned): inputs in, step, outputs out
    e2e = None
    if isinstance(work, DecodeStack) and not args.no_e2e:
        hx = torch.empty(work.x_all.shape, dtype=torch.bfloat16, pin_memory=True)
        hx.copy_(work.x_all)
        hq = torch.empty(work.y_qkv.shape, dtype=torch.float32, pin_memory=True)
        hy = torch.empty(work.y.shape, dtype=torch.float32, pin_memory=True)
        e_steps = max(3, min(args.steps, 50))
        with torch.cuda.stream(s):
            for _ in range(3):
                work.step_e2e(hx, hq, hy)
            if world > 1:
                torch.distributed.barrier()
            t0 = time.perf_counter()
            for _ in range(e_steps):
                work.step_e2e(hx, hq, hy)
            dt = (time.perf_counter() - t0) / e_steps
        if world > 1:
            t = torch.tensor([dt], device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            dt = float(t.item())
        e2e = {"value": round(work.bytes_per_step * world / dt / 1e9, 2), "unit": "GB/s",
               "h2d_bytes_per_step": hx.numel() * 2, "d2h_bytes_per_step": (hq.numel() + hy.numel()) * 4,
               "ms_per_step": round(dt * 1e3, 3), "steps": e_steps,
               "path": ("onpu_chain_run" if work.chain is not None else "onpu_dense_mv_dev")
               + " with pinned host input/output copies and a host synchronisation per step (wall clock)"}
        # the reference ABI's host-pointer call (onpu_dense_mv: fp32 host in/out, copies and a
        # synchronisation inside every call, SwiGLU on the host), as a second end-to-end figure
        xs = [np.ascontiguousarray(xl.float().cpu().numpy()) for xl in work.x]
        ys = {"qkv": np.empty((M, QKV_N), np.float32), "gate_up": np.empty((M, 2 * INTER), np.float32),
              "down": np.empty((M, HIDDEN), np.float32)}
        work.step_host(xs, ys)
        r_steps = max(2, min(args.steps, 5))
        t0 = time.perf_counter()
        for _ in range(r_steps):
            work.step_host(xs, ys)
        rt = (time.perf_counter() - t0) / r_steps
        e2e["reference_abi"] = {"value": round(work.bytes_per_step / rt / 1e9, 2), "unit": "GB/s",
                                "ms_per_step": round(rt * 1e3, 3), "path": "onpu_dense_mv per matrix (host fp32)",
                                "h2d_bytes_per_step": args.layers * M * (HIDDEN * 4 * 2 + INTER * 4),
                                "d2h_bytes_per_step": args.layers * M * (QKV_N + 2 * INTER + HIDDEN) * 4}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and isinstance(work, DecodeStack):
        dq, ss, cores, sample = cpu_reference_sample(M, seconds=args.cpu_seconds)
        cpu = {"value": round(dq, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample,
               "steady_state_prequantised_value": round(ss, 3)}

    traffic = None
    tp = ROOT / "profiles" / "traffic.json"
    if tp.exists():
        mode = args.mode if args.config == "qwen3-8b" else "launches"
        traffic = json.loads(tp.read_text()).get(f"{args.config}/{mode}")
    if rank == 0:
        achieved = dom_bytes / (dom_us * 1e-6) / 1e9
        line = {
            "metric": "int4 GEMV achieved HBM GB/s (Qwen3-8B decode projections, 36 layers)"
            if args.config == "qwen3-8b" else "int4 GEMV achieved HBM GB/s (4096x4096, M=1)",
            "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4xbf16->fp32", "data": "synthetic (seeded random int4 weights, fp16 scales, bf16 N(0,1))",
            "config": {"workload": "qwen3-8b-decode-projections" if args.config == "qwen3-8b" else "gemv-4096x4096",
                       "M": M, "layers": args.layers if args.config == "qwen3-8b" else 1,
                       "bytes_per_step_per_gpu": work.bytes_per_step,
                       "weight_bytes_per_step_per_gpu": work.weight_bytes_per_step,
                       "parallelism": f"replicas{world}", "l2": "inputs larger than L2 (no flush needed)",
                       "cuda_graph": graph is not None,
                       "mode": args.mode if args.config == "qwen3-8b" else "launches",
                       "mlp_activation": getattr(work, "act", None)},
            "tokens_per_s": round(M * world / (ms_step * 1e-3), 1) if args.config == "qwen3-8b" else None,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_kind": peak_kind, "traffic": traffic,
                         "kernel": dom_name, "algorithmic_bytes_per_launch": dom_bytes,
                         "us_per_launch": round(dom_us, 3)},
            "cpu_baseline": cpu, "e2e": e2e, "clocks": clk,
            "gpu_launches": work.launches_per_step * args.steps,
        }
        print(json.dumps(line), flush=True)
    if graph is not None:
        del graph
    if world > 1:
        torch.distributed.destroy_process_group()


def run_reference(args):
    """The reference's CPU implementation of the path (the oracle port: dequantise per 32, then
    fp32 torch matmul, all host threads) on the same config, metric and unit as our arm; each step
    is a bounded sample. Rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    M = args.m
    n_steps = args.warmup + args.steps
    per = max(0.2, min(1.0, 120.0 / n_steps))                # the whole arm stays near two minutes
    cfg = args.config
    vals, sample, cores, kind = [], None, None, "port"
    for i in range(n_steps):
        if cfg in ("qwen3-8b", "gemv"):
            v, _, cores, sample = cpu_reference_sample(M, seconds=per, seed=i)
        elif cfg == "prefill":
            v, cores, sample = cpu_prefill_sample(seconds=per)
        elif cfg == "moe":
            v, cores, sample = cpu_moe_sample(max(M, 1), seconds=per)
        elif cfg == "attn":
            v, cores, kind, sample = cpu_attn_sample(args.context, seconds=per, seed=i)
        else:
            gbs, cores, sample = cpu_tp_sample(M, seconds=per)
            from opennpu_b200 import tp
            step_bytes = args.layers * sum(int4_param_bytes(N, K)
                                           for _, N, K in tp.dense_layer_shapes(T_HIDDEN, T_INTER, T_QH, T_KVH))
            v = gbs * 1e9 / step_bytes * M
        if i >= args.warmup:
            vals.append(v)
    v = float(np.median(vals))
    metric, unit, workload = {
        "qwen3-8b": ("int4 GEMV achieved HBM GB/s (Qwen3-8B decode projections, 36 layers)", "GB/s",
                     "qwen3-8b-decode-projections"),
        "gemv": ("int4 GEMV achieved HBM GB/s (Qwen3-8B decode projections, 36 layers)", "GB/s",
                 "qwen3-8b-decode-projections"),
        "prefill": ("int4 prefill dequant-GEMM TFLOP/s (Qwen3-14B MLP, tcgen05)", "TFLOP/s", "qwen3-14b-prefill-mlp"),
        "moe": ("MoE layer tokens/s (Qwen3-30B-A3B: router + 128-expert top-8 int4 FFN)", "tokens/s",
                "qwen3-30b-a3b-moe-layer"),
        "qwen2.5-32b": ("int4 dense decode stack tokens/s (Qwen2.5-32B, tensor-parallel)", "tokens/s",
                        "qwen2.5-32b-decode-projections-tp"),
        "attn": ("decode attention KV-cache GB/s (Qwen3-8B, 36 layers, bf16 cache)", "GB/s",
                 "qwen3-8b-decode-attention"),
    }[cfg]
    line = {"impl": "reference", "metric": metric, "value": round(v, 4), "unit": unit,
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong" if cfg == "qwen2.5-32b" else "weak", "vs_baseline": None,
            "dtype": "bf16 cache, fp32 arithmetic" if cfg == "attn" else "int4 dequantised to fp32",
            "data": "synthetic",
            "config": (tp_config(M, args.layers, int(os.environ.get("WORLD_SIZE", "1"))) if cfg == "qwen2.5-32b"
                       else {"workload": workload, "M": M, "layers": args.layers,
                             **({"context": args.context} if cfg == "attn" else {})}),
            "cpu_baseline": {"value": round(v, 4), "unit": unit, "cores": cores, "kind": kind,
                             "sample": f"per step ({per:.2f} s): {sample}"},
            "e2e": {"value": round(v, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="qwen2.5-32b",
                    choices=["qwen2.5-32b", "qwen3-8b", "gemv", "prefill", "moe", "attn"])
    ap.add_argument("--context", type=int, default=4096, help="attn: KV-cache length (tokens)")
    ap.add_argument("--m", "--rows", dest="m", type=int, default=1,
                    help="tokens (M / T); spell it --rows under torchrun, which claims --m")
    ap.add_argument("--allreduce", default="peer", choices=["peer", "nccl"],
                    help="qwen2.5-32b at N>1: the row-parallel all-reduce (peer-memory kernel or NCCL)")
    ap.add_argument("--moe-fused", type=int, default=1, choices=[0, 1],
                    help="moe: the expert FFN as one persistent launch (1, default) or three launches (0); "
                         "onpu_moe_set_fused")
    ap.add_argument("--ep", default="gather", choices=["gather", "a2a"],
                    help="moe at N>1: all-gather + reduce-scatter (graph-captured) or all-to-all dispatch/combine")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="qwen2.5-32b: skip the Qwen3-8B figures at N = 1")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--act", default="f32", choices=["f32", "bf16"],
                    help="qwen3-8b: the MLP activation between gate/up and down (fp32, or rounded to bf16)")
    ap.add_argument("--mode", default="launches", choices=["chain", "launches"],
                    help="chain: the step as one persistent GEMV-chain launch; launches: one launch per matrix")
    ap.add_argument("--layers", type=int, default=None,
                    help="decoder layers in the stack (profiling captures use fewer; the metric is quoted at the "
                         "config's own count: qwen2.5-32b 64, qwen3-8b 36, moe 48)")
    args = ap.parse_args()
    if args.layers is None:
        args.layers = {"qwen2.5-32b": T_LAYERS, "qwen3-8b": LAYERS, "moe": M_LAYERS, "attn": A_LAYERS}.get(args.config, 1)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.config == "prefill":
        run_prefill(args)
    elif args.config == "moe":
        run_moe(args)
    elif args.config == "qwen2.5-32b":
        run_tp(args)
    elif args.config == "attn":
        run_attn(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
