"""Device-resident MoE layer: router and routed-expert FFN on torch CUDA tensors.

``route`` is the reference router (opennpu/native/reference.py:71-76): softmax over h . Wr^T,
top-k, weights renormalised over the k. ``ExpertFFN`` holds E experts' gate/up and down matrices
as int4 + fp16 scales (group 32) and runs y[t] = sum_j w[t, j] * down_e(silu(gate_e x_t) *
up_e x_t) with the grouped GEMV (one job per expert and up to 16 of its tokens), the SwiGLU fused
into the gate_up GEMV, and the weighted combine (reference.py:77-84).
"""
import torch

from . import libonpu as L
from .dense import _stream_ptr


def route(h, wr, k, norm_topk_prob=True, logits=False, stream=None):
    """h: bf16 CUDA [T, H], wr: bf16 CUDA [E, H] -> (ids int32 [T, k], w fp32 [T, k]) and, with
    ``logits``, the fp32 logits [T, E]. ids in descending probability, lower id first on ties."""
    assert h.is_cuda and h.dtype == torch.bfloat16 and h.dim() == 2 and h.stride(1) == 1
    assert wr.is_cuda and wr.dtype == torch.bfloat16 and wr.is_contiguous()
    T, E, H = h.shape[0], wr.shape[0], wr.shape[1]
    ids = torch.empty(T, k, dtype=torch.int32, device=h.device)
    w = torch.empty(T, k, dtype=torch.float32, device=h.device)
    lg = torch.empty(T, E, dtype=torch.float32, device=h.device) if logits else None
    rc = L.load().onpu_route_dev(h.data_ptr(), h.stride(0), T, wr.data_ptr(), E, H, k, int(norm_topk_prob),
                                 ids.data_ptr(), w.data_ptr(), 0 if lg is None else lg.data_ptr(),
                                 _stream_ptr(stream))
    L.check(rc, "onpu_route_dev")
    return (ids, w, lg) if logits else (ids, w)


class ExpertFFN:
    """E routed experts: gate_up [E, 2I, H] (gate rows then up rows) and down [E, H, I], each as
    int4 packed along K (uint8 [.., N, K/2]) plus fp16 scales [.., N, K/32]."""

    def __init__(self, gu_qk, gu_s, dn_qk, dn_s, stream=None):
        lib = L.require_device()
        E, Ng, Kg = gu_qk.shape[0], gu_qk.shape[1], gu_qk.shape[2] * 2
        Nd, Kd = dn_qk.shape[1], dn_qk.shape[2] * 2
        self.E, self.H, self.I, self.Nd = E, Kg, Ng // 2, Nd
        self.h = lib.onpu_ffn_new_int4(Ng, Kg, Nd, Kd, E)
        if not self.h:
            raise L.OnpuError(f"onpu_ffn_new_int4: {L.last_error()}")
        self._load(lib.onpu_ffn_gu(self.h), gu_qk, gu_s, stream)
        self._load(lib.onpu_ffn_dn(self.h), dn_qk, dn_s, stream)

    @staticmethod
    def _load(bank, qk, s, stream):
        lib = L.load()
        qk = qk.contiguous()
        s = s.contiguous().view(torch.int16) if s.dtype == torch.float16 else s.contiguous()
        if qk.is_cuda:
            rc = lib.onpu_bank_load_int4(bank, qk.data_ptr(), s.data_ptr(), 1, _stream_ptr(stream))
        else:
            rc = lib.onpu_bank_load_int4(bank, qk.numpy().ctypes.data, s.numpy().ctypes.data, 0, None)
        L.check(rc, "onpu_bank_load_int4")

    def __call__(self, x, ids, w, out=None, stream=None):
        """x: bf16 CUDA [T, H]; ids int32 / w fp32 CUDA [T, k] (from ``route``) -> fp32 [T, H]."""
        assert x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
        assert ids.dtype == torch.int32 and ids.is_contiguous() and w.dtype == torch.float32 and w.is_contiguous()
        T, k = ids.shape
        if out is None:
            out = torch.empty(T, self.Nd, dtype=torch.float32, device=x.device)
        rc = L.load().onpu_moe_ffn_dev(self.h, x.data_ptr(), x.stride(0), T, ids.data_ptr(), w.data_ptr(), k,
                                       out.data_ptr(), out.stride(0), _stream_ptr(stream))
        L.check(rc, "onpu_moe_ffn_dev")
        return out

    def __del__(self):
        try:
            if getattr(self, "h", None):
                L.load().onpu_ffn_free(self.h)
                self.h = None
        except Exception:   # interpreter shutdown: the library may already be unloaded
            pass
