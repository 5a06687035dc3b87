"""Device-resident dense int4 matrices driven with torch CUDA tensors (libonpu's _dev entry points).

``DenseMatrix`` owns one libonpu dense handle. Weights come from int4 packed along K (two's
complement, element 2j in the low nibble of byte j) with fp16 scales per 32 (``from_int4``), or
from the reference's stream-order upload buffer (``from_stream``, formats q4nx / q4s). ``mv``
runs y = x . W^T on the current torch stream, asynchronously.
"""
import numpy as np
import torch

from . import libonpu as L

EPI_F32, EPI_BF16, EPI_SWIGLU, EPI_PAIRSUM, EPI_SWIGLU_F32 = 0, 1, 2, 3, 5
FMT_Q4NX, FMT_Q4S, FMT_Q4F16 = 0, 1, 2


def _stream_ptr(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class DenseMatrix:
    def __init__(self, handle, N, K, fmt, gateup=False, residual=False):
        self.h, self.N, self.K, self.fmt, self.gateup, self.residual = handle, N, K, fmt, gateup, residual
        self.Kg = self.info()[2]          # K of the GPU layout (K rounded up to 32)

    # ---------------------------------------------------------------- construction
    @classmethod
    def from_int4(cls, qk, scales, gateup=False, stream=None):
        """qk: uint8 [N, K/2] packed int4, scales: fp16 (or its uint16 bits) [N, K/32]; CUDA or CPU
        tensors. gateup: rows [0, N/2) gate, [N/2, N) up (enables EPI_SWIGLU)."""
        lib = L.require_device()
        N, K = qk.shape[0], qk.shape[1] * 2
        h = lib.onpu_dense_new_int4(N, K, int(gateup))
        if not h:
            raise L.OnpuError(f"onpu_dense_new_int4: {L.last_error()}")
        m = cls(h, N, K, FMT_Q4F16, gateup)
        m.load_int4(qk, scales, stream)
        return m

    def load_int4(self, qk, scales, stream=None):
        lib = L.load()
        qk = qk.contiguous()
        sc = scales.contiguous().view(torch.int16) if scales.dtype == torch.float16 else scales.contiguous()
        on_dev = qk.is_cuda
        if on_dev:
            rc = lib.onpu_dense_load_int4(self.h, qk.data_ptr(), sc.data_ptr(), 1, _stream_ptr(stream))
        else:
            qn, sn = qk.numpy(), sc.numpy()
            rc = lib.onpu_dense_load_int4(self.h, qn.ctypes.data, sn.ctypes.data, 0, None)
        L.check(rc, "onpu_dense_load_int4")

    @classmethod
    def from_float(cls, W, sym=True, gateup=False, stream=None):
        """fp32 CUDA weights [N, K] quantised on the GPU with the reference's search quantisers
        (q4s when sym, else q4nx): the codes and scales the host packer would produce."""
        lib = L.require_device()
        assert W.is_cuda and W.dtype == torch.float32 and W.dim() == 2 and W.stride(1) == 1
        N, K = W.shape
        h = lib.onpu_dense_new_f32_dev(W.data_ptr(), W.stride(0), N, K, int(sym), int(gateup), _stream_ptr(stream))
        if not h:
            raise L.OnpuError(f"onpu_dense_new_f32_dev: {L.last_error()}")
        return cls(h, N, K, FMT_Q4S if sym else FMT_Q4NX, gateup)

    @classmethod
    def from_float_residual(cls, W, sym=True, stream=None):
        """The two-pass (~8-bit) form of fp32 CUDA weights [N, K] (N % 8 == 0): W and its
        quantisation residual, each quantised on the GPU, in one matrix of 2N GPU rows; ``mv`` with
        EPI_PAIRSUM (its default for these) returns the [M, N] sum of the two passes."""
        lib = L.require_device()
        assert W.is_cuda and W.dtype == torch.float32 and W.dim() == 2 and W.stride(1) == 1
        N, K = W.shape
        h = lib.onpu_dense_new_residual_f32_dev(W.data_ptr(), W.stride(0), N, K, int(sym), _stream_ptr(stream))
        if not h:
            raise L.OnpuError(f"onpu_dense_new_residual_f32_dev: {L.last_error()}")
        return cls(h, 2 * N, K, FMT_Q4S if sym else FMT_Q4NX, residual=True)

    # ---------------------------------------------------------------- weight blobs
    def export(self):
        """The matrix as a self-describing blob of its GPU layout (uint8 numpy array; the bytes a
        PackCache stores)."""
        return L.export_blob(L.load().onpu_dense_export, self.h, "onpu_dense_export")

    @classmethod
    def from_blob(cls, blob):
        """A matrix from an ``export`` blob: one host->device copy, no quantisation or repack."""
        lib = L.require_device()
        b = L.as_blob(blob)
        h = lib.onpu_dense_import(b.ctypes.data, b.size)
        if not h:
            raise L.OnpuError(f"onpu_dense_import: {L.last_error()}")
        sec = L.blob_sections(b)[1][0]
        return cls(h, sec["N"], sec["K"], sec["fmt"], gateup=sec["flags"] == L.BLOB_GATEUP,
                   residual=sec["flags"] == L.BLOB_RESIDUAL)

    @classmethod
    def from_stream(cls, N, K, sym, packed):
        """The reference upload protocol: onpu_dense_new2 + fill onpu_dense_buf + onpu_dense_sync."""
        lib = L.require_device()
        h = lib.onpu_dense_new2(N, K, int(sym))
        if not h:
            raise L.OnpuError(f"onpu_dense_new2: {L.last_error()}")
        nb = lib.onpu_dense_bytes(h)
        buf = np.ctypeslib.as_array(lib.onpu_dense_buf(h), shape=(nb,))
        buf[:] = np.asarray(packed, np.uint8)
        lib.onpu_dense_sync(h)
        if L.last_error():
            raise L.OnpuError(L.last_error())
        return cls(h, N, K, FMT_Q4S if sym else FMT_Q4NX)

    def __del__(self):
        try:
            if getattr(self, "h", None):
                L.load().onpu_dense_free(self.h)
                self.h = None
        except Exception:   # interpreter shutdown: the library may already be unloaded
            pass

    # ---------------------------------------------------------------- use
    def info(self):
        out = (L.C.c_int64 * 4)()
        L.load().onpu_dense_info(self.h, out)
        return tuple(out)

    @property
    def nbytes(self):
        return self.info()[3]

    def max_f32_rows(self):
        """The most activation rows (0..8) an fp32-input call takes for this matrix."""
        return int(L.load().onpu_dense_max_f32_rows(self.h))

    def prepare(self, rows):
        L.check(L.load().onpu_dense_prepare(self.h, rows), "onpu_dense_prepare")

    def mv(self, x, out=None, epi=None, stream=None):
        """x: bf16 CUDA [M, K] (row stride % 8 == 0), or fp32 [M <= 8, K] (row stride % 4 == 0; each
        value staged as two fp16 halves, so it is not rounded to 16 bits) -> [M, N] fp32 (EPI_F32),
        bf16 (EPI_BF16), [M, N/2] silu(gate) * up in bf16 (EPI_SWIGLU) or fp32 (EPI_SWIGLU_F32), or
        [M, N/2] fp32 row + residual (EPI_PAIRSUM, the default of a two-pass matrix; EPI_F32
        otherwise)."""
        assert x.is_cuda and x.dtype in (torch.bfloat16, torch.float32) and x.dim() == 2 and x.stride(1) == 1
        if epi is None:
            epi = EPI_PAIRSUM if self.residual else EPI_F32
        M = x.shape[0]
        if out is None:
            ncol = self.N // 2 if epi in (EPI_SWIGLU, EPI_SWIGLU_F32, EPI_PAIRSUM) else self.N
            fp32 = epi in (EPI_F32, EPI_PAIRSUM, EPI_SWIGLU_F32)
            out = torch.empty(M, ncol, device=x.device, dtype=torch.float32 if fp32 else torch.bfloat16)
        fn = "onpu_dense_mv_f32_dev" if x.dtype == torch.float32 else "onpu_dense_mv_dev"
        rc = getattr(L.load(), fn)(self.h, x.data_ptr(), x.stride(0), M, out.data_ptr(), out.stride(0), epi,
                                   _stream_ptr(stream))
        L.check(rc, fn)
        return out

    def mm(self, x, out=None, epi=EPI_F32, stream=None):
        """Many tokens (prefill) on the tensor cores: like ``mv`` for any number of rows, with the
        weights dequantised to fp16."""
        assert x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
        M = x.shape[0]
        if out is None:
            ncol = self.N // 2 if epi == EPI_SWIGLU else self.N
            out = torch.empty(M, ncol, device=x.device, dtype=torch.float32 if epi == EPI_F32 else torch.bfloat16)
        rc = L.load().onpu_dense_mm_dev(self.h, x.data_ptr(), x.stride(0), M, out.data_ptr(), out.stride(0), epi,
                                        _stream_ptr(stream))
        L.check(rc, "onpu_dense_mm_dev")
        return out

    def unpack(self):
        """GPU layout -> (codes uint8 [N, Kg], scale bits int16 [N, Kg/32], min bits or None), in GPU
        row order (a gate/up matrix is interleaved per 16 rows); Kg = K rounded up to 32."""
        dev = torch.device("cuda")
        q = torch.zeros(self.N, self.Kg, dtype=torch.uint8, device=dev)
        s = torch.zeros(self.N, self.Kg // 32, dtype=torch.int16, device=dev)
        m = torch.zeros_like(s) if self.fmt == FMT_Q4NX else None
        rc = L.load().onpu_dense_unpack_dev(self.h, q.data_ptr(), s.data_ptr(), 0 if m is None else m.data_ptr(),
                                            _stream_ptr())
        L.check(rc, "onpu_dense_unpack_dev")
        torch.cuda.synchronize()
        return q, s, m


class DenseChain:
    """A sequence of ``DenseMatrix`` GEMVs on fixed CUDA buffers, run as one persistent launch
    (``onpu_chain_*``). Keep the tensors passed to ``add`` alive while the chain is used."""

    def __init__(self):
        lib = L.require_device()
        self.h = lib.onpu_chain_new()
        if not self.h:
            raise L.OnpuError(f"onpu_chain_new: {L.last_error()}")
        self._keep = []

    def add(self, m, x, y, epi=EPI_F32, dep=-1):
        assert x.is_cuda and x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
        assert y.is_cuda and y.dim() == 2 and y.stride(1) == 1
        idx = L.load().onpu_chain_add(self.h, m.h, x.data_ptr(), x.stride(0), x.shape[0], y.data_ptr(), y.stride(0),
                                      epi, dep)
        L.check(idx, "onpu_chain_add")
        self._keep += [m, x, y]
        return idx

    def dep(self, link):
        return L.load().onpu_chain_link_dep(self.h, link)

    def info(self):
        out = (L.C.c_int64 * 4)()
        L.load().onpu_chain_info(self.h, out)
        return tuple(out)

    def prepare(self):
        L.check(L.load().onpu_chain_prepare(self.h), "onpu_chain_prepare")

    def run(self, stream=None):
        L.check(L.load().onpu_chain_run(self.h, _stream_ptr(stream)), "onpu_chain_run")

    def trace(self, on=True):
        """Record %globaltimer stamps of later runs: returns the int64 CUDA tensor
        [CTAs, links, 8] they go to (see onpu_chain_trace), or None when turned off."""
        if not on:
            L.load().onpu_chain_trace(self.h, None)
            self._trace = None
            return None
        self.prepare()
        ctas, links = self.info()[1], self.info()[0]
        self._trace = torch.zeros(ctas, links, 8, dtype=torch.int64, device="cuda")
        L.load().onpu_chain_trace(self.h, self._trace.data_ptr())
        return self._trace

    def __del__(self):
        try:
            if getattr(self, "h", None):
                L.load().onpu_chain_free(self.h)
                self.h = None
        except Exception:
            pass


def check_device():
    """Synchronise and raise if a kernel reported a timed-out wait."""
    L.check(L.load().onpu_check_device(), "device status")
