"""Per-CTA timeline of the GEMV launches of a decode step, from the kernels' %globaltimer stamps.

    python -m opennpu_b200.gemv_timeline [layers] [M]

Runs `layers` layers of the Qwen3-8B decode projections (q/k/v 6144x4096, gate_up 24576x4096 with
the SwiGLU epilogue, down 4096x12288; random int4 weights) from a CUDA graph with tracing on
(onpu_gemv_trace, one stamp buffer per launch), and prints for each launch, in microseconds from
the first launch's first CTA: the spread of CTA entry times, the medians (relative to each CTA's
entry) of the producer's first weight copy, the consumers passing griddepcontrol.wait, the
activations staged and the first weights consumed, the spread of loop ends, the flush (row-group
close) times and the time the consumers waited for weights.
"""
import sys

import numpy as np
import torch

from . import libonpu as L
from .dense import DenseMatrix, EPI_F32, EPI_SWIGLU


def _mat(N, K, gen, gateup=False):
    qk = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=gen)
    s = (torch.randn(N, K // 32, device="cuda", generator=gen).abs() * 0.02 + 1e-4).half()
    return DenseMatrix.from_int4(qk, s, gateup=gateup)


def main(layers=4, M=1):
    lib = L.require_device()
    gen = torch.Generator(device="cuda").manual_seed(0)
    mats = [(_mat(6144, 4096, gen), _mat(24576, 4096, gen, True), _mat(4096, 12288, gen)) for _ in range(layers)]
    x = torch.randn(M, 4096, device="cuda", generator=gen).bfloat16()
    yq = torch.empty(M, 6144, device="cuda")
    a = torch.empty(M, 12288, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(M, 4096, device="cuda")
    ctas = torch.cuda.get_device_properties(0).multi_processor_count * 4
    bufs = [torch.zeros(ctas, 8, dtype=torch.int64, device="cuda") for _ in range(3 * layers)]
    s = torch.cuda.Stream()

    def step(trace):
        i = 0
        for q, gu, dn in mats:
            for m, xin, out, epi in ((q, x, yq, EPI_F32), (gu, x, a, EPI_SWIGLU), (dn, a, y, EPI_F32)):
                if trace:
                    lib.onpu_gemv_trace(bufs[i].data_ptr(), ctas)
                m.mv(xin, out=out, epi=epi, stream=s)
                i += 1
        lib.onpu_gemv_trace(None, 0)

    with torch.cuda.stream(s):
        step(False)
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        step(True)
    for _ in range(5):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    with torch.cuda.stream(s):
        for _ in range(20):
            graph.replay()
    e1.record(s)
    e1.synchronize()
    print(f"step {e0.elapsed_time(e1) / 20 * 1000:.1f} us for {layers} layers (with tracing)")
    with torch.cuda.stream(s):
        graph.replay()
    torch.cuda.synchronize()
    names = ["qkv", "gate_up", "down"]
    t0, prev_end = None, None
    for i, b in enumerate(bufs):
        t = b.cpu().numpy().astype(np.int64)
        t = t[t[:, 0] != 0]
        if t0 is None:
            t0 = t[:, 0].min()
        rel = (t[:, :7] - t0) / 1000.0
        ent, pro, pdl, stg, first, loop, fl = [rel[:, k] for k in range(7)]
        gap = "" if prev_end is None else f" gap_from_prev_end={ent.min() - prev_end:6.2f}"
        print(f"{i:2d} {names[i % 3]:8s} W={len(t):3d} entry[{ent.min():7.2f},{ent.max():7.2f}] "
              f"prod_issue_med={np.median(pro - ent):5.2f} pdl_med={np.median(pdl - ent):5.2f} "
              f"staged_med={np.median(stg - ent):5.2f} first_w_med={np.median(first - ent):5.2f} "
              f"loop_end[{loop.min():7.2f},{np.median(loop):7.2f},{loop.max():7.2f}] "
              f"flush_end_max={fl.max():7.2f} flush_med={np.median(fl - loop):5.2f} "
              f"flush_max={np.max(fl - loop):5.2f} waited_med={np.median(t[:, 7] / 1000.0):5.2f}{gap}")
        prev_end = fl.max()
    del graph


if __name__ == "__main__":
    main(*(int(a) for a in sys.argv[1:3]))
