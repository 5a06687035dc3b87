"""One-shot all-reduce of small fp32 vectors over NVLink peer memory (libonpu onpu_comm_*), for
the row-parallel projections of tensor-parallel decode: one launch per call, every rank writes its
partial into every peer's buffer and adds the world partials in rank order. The IPC handles are
exchanged over the torch.distributed process group once, at construction."""
import ctypes as C

import torch

from . import libonpu as L
from .dense import _stream_ptr


class PeerAllReduce:
    def __init__(self, group=None, cap_floats=1 << 16):
        dist = torch.distributed
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        lib = L.require_device()
        self.h = lib.onpu_comm_new(self.rank, self.world, cap_floats)
        if not self.h:
            raise L.OnpuError(f"onpu_comm_new: {L.last_error()}")
        self.cap = cap_floats
        mine = (C.c_ubyte * 64)()
        L.check(lib.onpu_comm_ipc_handle(self.h, mine), "onpu_comm_ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(mine), group=group)
        allh = (C.c_ubyte * (64 * self.world)).from_buffer_copy(b"".join(handles))
        L.check(lib.onpu_comm_open(self.h, allh), "onpu_comm_open")
        dist.barrier(group=group)        # every rank's buffer is mapped before the first call

    def __call__(self, t, out=None, out_bf16=None, stream=None):
        """t: fp32 CUDA contiguous; out (fp32, default: t in place unless only out_bf16 is given)
        and / or out_bf16 (bf16) receive the sum over ranks. Returns out, else out_bf16."""
        assert t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()
        if out is None and out_bf16 is None:
            out = t
        for o, dt in ((out, torch.float32), (out_bf16, torch.bfloat16)):
            assert o is None or (o.dtype == dt and o.is_contiguous() and o.numel() == t.numel())
        rc = L.load().onpu_comm_allreduce(self.h, t.data_ptr(), 0 if out is None else out.data_ptr(),
                                          0 if out_bf16 is None else out_bf16.data_ptr(), t.numel(),
                                          _stream_ptr(stream))
        L.check(rc, "onpu_comm_allreduce")
        return out if out is not None else out_bf16

    def close(self):
        if getattr(self, "h", None):
            L.load().onpu_comm_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:   # interpreter shutdown
            pass

    site = None                  # (N, K, rows, dtype) of the fused calls on this communicator

    def linear(self, m, x, out=None, out_bf16=None, stream=None):
        """The row-parallel projection fused with this all-reduce, one launch: the sum over ranks of
        x . W_rank^T for this rank's DenseMatrix shard m; the GEMV's epilogue sends its outputs to
        the peers and each CTA then sums every rank's words of its own rows. x: bf16 [M, K_rank], or
        fp32 [M <= 8, K_rank] (staged as two fp16 halves per value); out fp32 and / or out_bf16
        bf16 [M, N]. Every call on one communicator has the same shape (one per call site)."""
        assert x.is_cuda and x.dtype in (torch.bfloat16, torch.float32) and x.dim() == 2 and x.stride(1) == 1
        M = x.shape[0]
        if out is None and out_bf16 is None:
            out = torch.empty(M, m.N, device=x.device)
        for o, dt in ((out, torch.float32), (out_bf16, torch.bfloat16)):
            assert o is None or (o.dtype == dt and o.is_contiguous() and o.shape == (M, m.N))
        site = (m.N, m.K, M, x.dtype)
        if self.site is None:
            self.site = site
        elif self.site != site:                 # each CTA sums rows fixed by the shape: one site per handle
            raise ValueError(f"this communicator serves {self.site}; use another one for {site}")
        fn = "onpu_dense_mv_allreduce_f32_dev" if x.dtype == torch.float32 else "onpu_dense_mv_allreduce_dev"
        rc = getattr(L.load(), fn)(m.h, self.h, x.data_ptr(), x.stride(0), M, 0 if out is None else out.data_ptr(),
                                   0 if out_bf16 is None else out_bf16.data_ptr(), _stream_ptr(stream))
        L.check(rc, fn)
        return out if out is not None else out_bf16
