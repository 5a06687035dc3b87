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

    def export(self):
        """Both banks as one self-describing blob of their GPU layout (uint8 numpy array)."""
        return L.export_blob(L.load().onpu_ffn_export, self.h, "onpu_ffn_export")

    @classmethod
    def from_blob(cls, blob):
        """An FFN from an ``export`` blob: one host->device copy per bank, no repack."""
        lib = L.require_device()
        b = L.as_blob(blob)
        h = lib.onpu_ffn_import(b.ctypes.data, b.size)
        if not h:
            raise L.OnpuError(f"onpu_ffn_import: {L.last_error()}")
        gu, dn = L.blob_sections(b)[1]
        f = cls.__new__(cls)
        f.h, f.E, f.H, f.I, f.Nd = h, gu["E"], gu["K"], gu["N"] // 2, dn["N"]
        return f

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

    def __call__(self, x, ids, w, out=None, stream=None, e0=None):
        """x: bf16 CUDA [T, H]; ids int32 / w fp32 CUDA [T, k] (from ``route``) -> fp32 [T, H].
        e0: this FFN holds experts e0 .. e0 + E - 1 of a larger pool (expert parallelism); slots
        routed elsewhere are skipped and the result is this shard's share of the sum."""
        assert x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
        assert ids.dtype == torch.int32 and ids.is_contiguous() and w.dtype == torch.float32 and w.is_contiguous()
        T, k = ids.shape
        if out is None:
            out = torch.empty(T, self.Nd, dtype=torch.float32, device=x.device)
        lib = L.load()
        if e0 is None:
            rc = lib.onpu_moe_ffn_dev(self.h, x.data_ptr(), x.stride(0), T, ids.data_ptr(), w.data_ptr(), k,
                                      out.data_ptr(), out.stride(0), _stream_ptr(stream))
        else:
            rc = lib.onpu_moe_ffn_dev_ep(self.h, x.data_ptr(), x.stride(0), T, ids.data_ptr(), w.data_ptr(), k, e0,
                                         out.data_ptr(), out.stride(0), _stream_ptr(stream))
        L.check(rc, "onpu_moe_ffn_dev")
        return out

    def layer(self, x, wr, k=8, norm_topk_prob=True, out=None, ids=None, w=None, stream=None):
        """The whole layer in one call (onpu_moe_layer_dev): route x with the bf16 router matrix wr
        [E, H] (the job lists are built by the router's last CTA), then the experts. Returns
        (y fp32 [T, H], ids int32 [T, k], w fp32 [T, k])."""
        assert x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
        assert wr.is_cuda and wr.dtype == torch.bfloat16 and wr.is_contiguous() and wr.shape == (self.E, self.H)
        T = x.shape[0]
        ids = torch.empty(T, k, dtype=torch.int32, device=x.device) if ids is None else ids
        w = torch.empty(T, k, device=x.device) if w is None else w
        out = torch.empty(T, self.Nd, device=x.device) if out is None else out
        rc = L.load().onpu_moe_layer_dev(self.h, wr.data_ptr(), x.data_ptr(), x.stride(0), T, k, int(norm_topk_prob),
                                         ids.data_ptr(), w.data_ptr(), out.data_ptr(), out.stride(0),
                                         _stream_ptr(stream))
        L.check(rc, "onpu_moe_layer_dev")
        return out, ids, w

    def __del__(self):
        try:
            if getattr(self, "h", None):
                L.load().onpu_ffn_free(self.h)
                self.h = None
        except Exception:   # interpreter shutdown: the library may already be unloaded
            pass


class EPMoELayer:
    """Expert-parallel MoE layer on one rank of a process group (NCCL): this rank holds experts
    [rank * E / world, (rank + 1) * E / world) and its own T tokens. The ranks all-gather their
    tokens and routing (ids, weights), each runs its experts over every rank's tokens routed to
    them, and a reduce-scatter sums the shares back to the tokens' owners. The router runs where
    the tokens live."""

    def __init__(self, wr, ffn, rank, world, E, group=None, k=8, norm_topk_prob=True):
        self.wr, self.ffn, self.rank, self.world, self.group = wr, ffn, rank, world, group
        self.E, self.k, self.norm = E, k, norm_topk_prob
        assert E % world == 0 and ffn.E == E // world
        self.e0 = rank * (E // world)

    def buffers(self, T, H, device="cuda"):
        W = self.world
        return {"ids": torch.empty(T, self.k, dtype=torch.int32, device=device),
                "w": torch.empty(T, self.k, device=device),
                "x_all": torch.empty(W * T, H, dtype=torch.bfloat16, device=device),
                "ids_all": torch.empty(W * T, self.k, dtype=torch.int32, device=device),
                "w_all": torch.empty(W * T, self.k, device=device),
                "y_all": torch.empty(W * T, self.ffn.Nd, device=device),
                "y": torch.empty(T, self.ffn.Nd, device=device)}

    def __call__(self, x, b, stream=None):
        """x: bf16 [T, H] (this rank's tokens) -> b["y"] fp32 [T, H]."""
        T = x.shape[0]
        lib = L.load()
        rc = lib.onpu_route_dev(x.data_ptr(), x.stride(0), T, self.wr.data_ptr(), self.E, self.wr.shape[1], self.k,
                                int(self.norm), b["ids"].data_ptr(), b["w"].data_ptr(), None, _stream_ptr(stream))
        L.check(rc, "onpu_route_dev")
        dist = torch.distributed
        dist.all_gather_into_tensor(b["x_all"], x, group=self.group)
        dist.all_gather_into_tensor(b["ids_all"], b["ids"], group=self.group)
        dist.all_gather_into_tensor(b["w_all"], b["w"], group=self.group)
        self.ffn(b["x_all"], b["ids_all"], b["w_all"], out=b["y_all"], stream=stream, e0=self.e0)
        dist.reduce_scatter_tensor(b["y"], b["y_all"], group=self.group)
        return b["y"]


def plan_dispatch(ids, E, world):
    """Which of a rank's tokens go to which rank: rank d holds experts [d * E / world, (d + 1) * E /
    world); a token goes to every rank holding one of its k experts, once. Returns (order, counts):
    order int64 [S] lists token indices grouped by destination rank (ascending token order within
    each), counts int64 [world] the tokens per destination (S = counts.sum())."""
    T = ids.shape[0]
    dest = (ids.long() // (E // world))                                   # [T, k]
    hit = torch.zeros(T, world, dtype=torch.bool, device=ids.device)
    hit.scatter_(1, dest, True)
    counts = hit.sum(0)
    order = hit.t().nonzero()[:, 1]                                       # rank-major, then token
    return order, counts


class EPMoELayerA2A:
    """Expert-parallel MoE layer with an all-to-all dispatch and combine (NCCL): each rank routes
    its own T tokens and sends every token only to the ranks that hold one of its experts (with its
    ids and weights); each rank runs its experts over the tokens it received (the slots routed to
    other ranks are skipped) and sends each token's share back; the owner adds the shares in rank
    order. Against EPMoELayer's all-gather / reduce-scatter this moves only the rows a rank needs,
    but the counts are exchanged first and read on the host (split sizes), so a call is not
    capturable in a CUDA graph."""

    def __init__(self, wr, ffn, rank, world, E, group=None, k=8, norm_topk_prob=True):
        self.wr, self.ffn, self.rank, self.world, self.group = wr, ffn, rank, world, group
        self.E, self.k, self.norm = E, k, norm_topk_prob
        assert E % world == 0 and ffn.E == E // world
        self.e0 = rank * (E // world)

    def __call__(self, x, stream=None):
        """x: bf16 [T, H] (this rank's tokens) -> fp32 [T, H]."""
        dist = torch.distributed
        T, H = x.shape
        ids, w = route(x, self.wr, self.k, self.norm, stream=stream)
        order, counts = plan_dispatch(ids, self.E, self.world)
        recv_counts = torch.empty_like(counts)
        dist.all_to_all_single(recv_counts, counts, group=self.group)
        send_sizes, recv_sizes = counts.tolist(), recv_counts.tolist()    # host: the split sizes
        R = sum(recv_sizes)
        xs, ids_s, w_s = x[order].contiguous(), ids[order].contiguous(), w[order].contiguous()
        xr = torch.empty(R, H, dtype=x.dtype, device=x.device)
        ids_r = torch.empty(R, self.k, dtype=ids.dtype, device=x.device)
        w_r = torch.empty(R, self.k, dtype=w.dtype, device=x.device)
        dist.all_to_all_single(xr, xs, recv_sizes, send_sizes, group=self.group)
        dist.all_to_all_single(ids_r, ids_s, recv_sizes, send_sizes, group=self.group)
        dist.all_to_all_single(w_r, w_s, recv_sizes, send_sizes, group=self.group)
        yr = self.ffn(xr, ids_r, w_r, stream=stream, e0=self.e0) if R else torch.empty(0, H, device=x.device)
        yb = torch.empty(order.numel(), yr.shape[1], dtype=yr.dtype, device=x.device)
        dist.all_to_all_single(yb, yr, send_sizes, recv_sizes, group=self.group)
        y = torch.zeros(T, yr.shape[1], dtype=yr.dtype, device=x.device)
        o = 0
        for n in send_sizes:                      # rank order: the same float sums on every run
            if n:
                y.index_add_(0, order[o:o + n], yb[o:o + n])
            o += n
        return y
