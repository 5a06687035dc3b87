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
