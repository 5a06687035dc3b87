"""Decode attention on a KV cache resident in HBM (onpu_attn_step_dev): one token of softmax
attention for every query head, GQA heads sharing their kv head's cache rows, with the
reference's additive mask and per-head sinks (llama/ggml-opennpu/onpu_cpu.cpp:173-229)."""
import torch

from . import libonpu as L


def attn_step(q, k, v, mask=None, sinks=None, scale=None, out=None, stream=None):
    """q: fp32 CUDA [Hq, D]; k, v: fp32 or bf16 CUDA [Hkv, S, D] views with unit stride along D
    (a cache slice [Hkv, :S, D] keeps its head stride); mask fp32 [S] or None; sinks fp32 [Hq] or
    None; scale defaults to D ** -0.5. Returns fp32 [Hq, D]."""
    assert q.is_cuda and q.dtype == torch.float32 and q.dim() == 2 and q.is_contiguous()
    assert k.shape == v.shape and k.stride() == v.stride() and k.dim() == 3 and k.stride(2) == 1
    assert k.dtype == v.dtype and k.dtype in (torch.float32, torch.bfloat16)
    Hq, D = q.shape
    Hkv, S, _ = k.shape
    for t, n in ((mask, S), (sinks, Hq)):
        assert t is None or (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous() and t.numel() == n)
    out = torch.empty(Hq, D, device=q.device) if out is None else out
    s = stream if stream is not None else torch.cuda.current_stream()
    rc = L.require_device().onpu_attn_step_dev(
        q.data_ptr(), Hq, D, k.data_ptr(), v.data_ptr(), Hkv, S, k.stride(0), k.stride(1),
        None if mask is None else mask.data_ptr(), None if sinks is None else sinks.data_ptr(),
        float(D ** -0.5 if scale is None else scale), out.data_ptr(), int(k.dtype == torch.bfloat16), s.cuda_stream)
    L.check(rc, "onpu_attn_step_dev")
    return out


def _main():
    """Time onpu_attn_step_dev: CUDA events over many calls queued behind a GPU sleep (so the
    host's call rate does not bound them), distinct caches per call so the working set exceeds
    the L2. Prints one JSON line per shape: microseconds per call and cache GB/s."""
    import argparse
    import json
    ap = argparse.ArgumentParser(description=_main.__doc__)
    ap.add_argument("--shapes", nargs="*", default=["32,8,128,4096,bf16", "32,8,128,32768,bf16",
                                                    "40,8,128,8192,bf16", "64,8,64,8192,f32"],
                    help="Hq,Hkv,D,S,dtype (bf16 or f32)")
    ap.add_argument("--caches", type=int, default=16)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    for spec in a.shapes:
        Hq, Hkv, D, S, dt = spec.split(",")
        Hq, Hkv, D, S = int(Hq), int(Hkv), int(D), int(S)
        dtype = torch.bfloat16 if dt == "bf16" else torch.float32
        g = torch.Generator(device="cuda").manual_seed(S)
        q = torch.randn(Hq, D, device="cuda", generator=g)
        ks = [torch.randn(Hkv, S, D, device="cuda", generator=g).to(dtype) for _ in range(a.caches)]
        vs = [torch.randn(Hkv, S, D, device="cuda", generator=g).to(dtype) for _ in range(a.caches)]
        out = torch.empty(Hq, D, device="cuda")
        for _ in range(a.warmup):
            for k, v in zip(ks, vs):
                attn_step(q, k, v, out=out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(200_000_000)
        e0.record()
        for _ in range(a.iters):
            for k, v in zip(ks, vs):
                attn_step(q, k, v, out=out)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (a.iters * a.caches)
        nbytes = 2 * Hkv * S * D * ks[0].element_size()
        print(json.dumps(dict(Hq=Hq, Hkv=Hkv, D=D, S=S, cache=dt, us_per_call=round(us, 2),
                              cache_GBs=round(nbytes / us / 1e3, 1), launches_per_call=2)))
        del ks, vs


if __name__ == "__main__":
    _main()
