"""The reference's 4-bit engine call shapes (opennpu/native/npu4/model.py), backed by libonpu for B200.

Same names, arguments and behaviour as the reference's classes for the int4 matmul path:

- ``Mat``             geometry of a packed matrix (model.py:151-255; opennpu_core.hpp:65-97)
- ``quant_sym``       numpy q4s quantiser (model.py:127-147)
- ``clib``            the ctypes libonpu (model.py:281-335) - here the B200 library
- ``quant_dequant``   what the device makes of W (model.py:343-350)
- ``check_geometry``  C geometry == Python geometry (model.py:353-360)
- ``NPULinearGroup``  sibling Linears packed as one matrix, one call for all (model.py:789-862)
- ``NPULinear``       nn.Module view of one sibling (model.py:865-880)
- ``NPUExperts``      a routed expert bank (model.py:883-1089), forward(hidden, indices, weights)
- ``expert_cols``     columns per expert (model.py:1174-1184)

Differences, all deliberate: no pyxrt fallback (no NPU here; without a B200 the constructors
raise), no PackCache disk cache and no vision / HIPREC paths (outside the int4 matmul path).
"""
import ctypes as C

import numpy as np
import torch
from torch import nn

from . import libonpu as L

NC, NR, GN, GK, KMAX = 8, 4, 64, 256, 2048
PKT = GN * GK // 2 + 2 * 2 * (GK // 32) * GN          # q4nx packet bytes
PKT_S = GN * GK // 2 + 2 * (GK // 32) * GN            # q4s packet bytes


def col_bytes(tiles, kc, sym=False):
    return tiles * kc * NR * (PKT_S if sym else PKT)


def _bf16_round(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint32) << 16
    return r.view(np.float32)


def quant_sym(W, group=32):
    """q4s: per 32 columns w ~= (q - 8) * d, q in 0..15, d bf16-exact; of 5 scales around
    absmax/8 the least squared error wins. Returns (codes uint8 [N, K], d float32 [N, K/32])."""
    N, K = W.shape
    g = W.reshape(N, K // group, group)
    peak = np.take_along_axis(g, np.abs(g).argmax(2)[..., None], 2)[..., 0]
    best = None
    for div in (-8.0, -7.5, -7.0, 7.0, 7.5):
        d = _bf16_round(np.asarray(peak / div, np.float32))
        d = np.where(d == 0, 1.0, d).astype(np.float32)
        v = np.clip(np.rint(g / d[..., None]), -8, 7)
        err = ((v * d[..., None] - g) ** 2).sum(2)
        if best is None:
            best = [v, d, err]
        else:
            better = err < best[2]
            best = [np.where(better[..., None], v, best[0]), np.where(better, d, best[1]), np.minimum(err, best[2])]
    return (best[0] + 8).astype(np.uint8).reshape(N, K), best[1]


class Mat:
    """Geometry of an [N, K] matrix on `ncols` reference device columns: R row blocks x S K-slices,
    (tiles, kc) packets each. It defines the size and byte order of the upload buffers
    (onpu_dense_buf / onpu_bank_buf); the B200 kernels themselves are shape-generic."""

    def __init__(self, N, K, ncols, sym=False):
        self.N, self.K, self.ncols, self.sym = N, K, ncols, sym
        best = None
        for S in [d for d in range(1, ncols + 1) if ncols % d == 0]:
            kc = -(-K // (S * GK))
            if kc > KMAX // GK:
                continue
            R = ncols // S
            tiles = -(-N // (R * NR * GN))
            if (tiles * kc) % 2:
                if kc + 1 <= KMAX // GK and tiles * (kc + 1) < (tiles + 1) * kc:
                    kc += 1
                else:
                    tiles += 1
            cost = (R * S * tiles * kc * (1 + 0.03 * (S - 1)), S)
            if best is None or cost < best[0]:
                best = (cost, R, S, tiles, kc)
        if best is None:
            raise ValueError(f"[{N}, {K}] needs more than {ncols} columns of K <= {KMAX}")
        _, self.R, self.S, self.tiles, self.kc = best
        self.ks = self.kc * GK
        self.rows_col = NR * self.tiles * GN
        self.cb = col_bytes(self.tiles, self.kc, sym)
        self.nbytes = self.R * self.S * self.cb

    def shapes(self):
        return {(self.tiles, self.kc)}

    def pack(self, W, threads=1):
        """W [N, K] float -> stream-order bytes, quantised by libonpu's search quantisers."""
        W = np.ascontiguousarray(W, np.float32)
        out = np.empty(self.nbytes, np.uint8)
        n = L.load().onpu_pack(L.fp(W), self.N, self.K, self.ncols, int(self.sym), out.ctypes.data_as(L.U8P), threads)
        if n != self.nbytes:
            raise RuntimeError(f"onpu_pack returned {n}, expected {self.nbytes}")
        return out


def clib():
    """libonpu with a usable B200 (raises otherwise: no CPU fallback)."""
    return L.require_device()


def quant_dequant(W, sym=False):
    W = np.ascontiguousarray(W, np.float32)
    out = np.empty_like(W)
    L.load().onpu_quant_dequant(L.fp(W), W.shape[0], W.shape[1], int(sym), L.fp(out), 8)
    return out


def check_geometry(m):
    out = (C.c_int64 * 8)()
    L.load().onpu_geometry2(m.N, m.K, m.ncols, int(m.sym), out)
    want = (m.R, m.S, m.tiles, m.kc, m.ks, m.rows_col, m.cb, m.nbytes)
    if tuple(out) != want:
        raise RuntimeError(f"libonpu geometry {tuple(out)} != {want}")


def expert_cols(topk, N=None, K=None):
    c = NC // topk if topk <= NC and NC % topk == 0 else 1
    while N is not None and c < NC:
        try:
            Mat(N, K, c)
            break
        except ValueError:
            c *= 2
    return c


def _upload(buf_ptr, nbytes):
    return np.ctypeslib.as_array(buf_ptr, shape=(nbytes,))


class NPULinearGroup:
    """Sibling Linear layers reading the same input, packed as one matrix: the first call computes
    all of them for that input, the others take their slice (model.py:789-862)."""

    def __init__(self, names, weights, sizes=None, K=None, sym=False, packed=None, residual=False):
        """weights: the matrices (or a callable returning them). packed: already-packed stream-order
        bytes (skips quantisation). residual: rows [W; W - quant_dequant(W)] (two 4-bit passes,
        ~8-bit precision), the two halves added after each product (model.py:793-833)."""
        self.names = names
        self.sizes = sizes or [w.shape[0] for w in weights]
        self.N1 = sum(self.sizes)
        self.residual = residual
        if K is None:
            K = (weights() if callable(weights) else weights)[0].shape[1]
        self.m = Mat(self.N1 * (2 if residual else 1), K, NC, sym)
        lib = clib()
        check_geometry(self.m)
        self.ch = lib.onpu_dense_new2(self.m.N, self.m.K, int(sym))
        if not self.ch:
            raise L.OnpuError(f"onpu_dense_new2: {L.last_error()}")
        buf = _upload(lib.onpu_dense_buf(self.ch), self.m.nbytes)
        if packed is None:
            ws = weights() if callable(weights) else weights
            W = np.ascontiguousarray(np.concatenate(ws) if len(ws) > 1 else ws[0], np.float32)
            if residual:
                W = np.concatenate([W, W - quant_dequant(W, sym)])
            packed = self.m.pack(W, threads=8)
        buf[:] = packed
        lib.onpu_dense_sync(self.ch)
        if L.last_error():
            raise L.OnpuError(L.last_error())
        self._key, self._y = None, None

    def __del__(self):
        try:
            if getattr(self, "ch", None):
                L.load().onpu_dense_free(self.ch)
                self.ch = None
        except Exception:
            pass

    def compute(self, x, i):
        if self._key is None or self._key[0] is not x or self._key[1] != x._version:
            xf = np.ascontiguousarray(x.detach().reshape(-1, x.shape[-1]).float().cpu().numpy())
            self._y = np.empty((len(xf), self.m.N), np.float32)
            clib().onpu_dense_mv(self.ch, L.fp(xf), len(xf), L.fp(self._y))
            err = L.last_error()
            if err:
                raise L.OnpuError(err)
            if self.residual:
                self._y = self._y[:, :self.N1] + self._y[:, self.N1:]
            self._key = (x, x._version)
        o = sum(self.sizes[:i])
        return self._y[:, o:o + self.sizes[i]]

    def full(self, x):
        self.compute(x, 0)
        return self._y


class NPULinear(nn.Module):
    def __init__(self, group, i, in_features, out_features, bias):
        super().__init__()
        self.group, self.i = group, i
        self.in_features, self.out_features = in_features, out_features
        self.bias = nn.Parameter(bias, requires_grad=False) if bias is not None else None

    def forward(self, x):
        shp = x.shape
        y = torch.from_numpy(np.ascontiguousarray(self.group.compute(x, self.i)))
        if self.bias is not None:
            y = y + self.bias.float()
        return y.to(x.dtype).reshape(*shp[:-1], self.out_features)

    def extra_repr(self):
        return f"{self.in_features} -> {self.out_features}, int4 on the B200"


class NPUExperts(nn.Module):
    """A 3-D expert bank on the B200. forward(hidden [T, H], indices [T, k], weights [T, k]) like
    the modules it replaces. gu[e]: [2I, H] ([gate | up] rows; gpt-oss: interleaved with
    act_kind 1), dn[e]: [H, I]."""

    def __init__(self, gu, dn, topk, gu_bias=None, dn_bias=None, sym=False, act_kind=0, alpha=1.702, limit=7.0,
                 packed=None):
        super().__init__()
        self.E, self.topk = len(gu) if packed is None else packed[0].shape[0], topk
        gs = gu[0].shape if packed is None else packed[2]
        ds = dn[0].shape if packed is None else packed[3]
        self.mgu = Mat(*gs, expert_cols(topk, *gs), sym)
        self.mdn = Mat(*ds, expert_cols(topk, *ds), sym)
        self.gu_bias = None if gu_bias is None else np.ascontiguousarray(gu_bias, np.float32)
        self.dn_bias = None if dn_bias is None else np.ascontiguousarray(dn_bias, np.float32)
        self.act_kind, self.alpha, self.limit = act_kind, float(alpha), float(limit)
        lib = clib()
        check_geometry(self.mgu)
        check_geometry(self.mdn)
        self.cffn = None
        if act_kind == 0 and gu_bias is None and dn_bias is None and self.mgu.ncols == 1 and self.mdn.ncols == 1:
            f = lib.onpu_ffn_new(self.mgu.N, self.mgu.K, self.mdn.N, self.mdn.K, self.E, int(sym))
            if f and lib.onpu_ffn_fused(f):
                self.cffn, self.cgu, self.cdn = f, lib.onpu_ffn_gu(f), lib.onpu_ffn_dn(f)
                perm = np.empty(self.mgu.N, np.int32)
                lib.onpu_ffn_perm(f, L.i32p(perm))
                self.perm = None if np.array_equal(perm, np.arange(self.mgu.N)) else perm
            elif f:
                lib.onpu_ffn_free(f)
        if self.cffn is None:
            self.perm = None
            self.cgu = lib.onpu_bank_new2(self.mgu.N, self.mgu.K, self.E, self.mgu.ncols, int(sym))
            self.cdn = lib.onpu_bank_new2(self.mdn.N, self.mdn.K, self.E, self.mdn.ncols, int(sym))
        if not (self.cgu and self.cdn):
            raise L.OnpuError(f"expert bank: {L.last_error()}")
        vg = np.ctypeslib.as_array(lib.onpu_bank_buf(self.cgu), shape=(self.E, self.mgu.nbytes))
        vd = np.ctypeslib.as_array(lib.onpu_bank_buf(self.cdn), shape=(self.E, self.mdn.nbytes))
        for e in range(self.E):
            if packed is not None:
                vg[e], vd[e] = packed[0][e], packed[1][e]
            else:
                g = gu[e] if self.perm is None else np.asarray(gu[e])[self.perm]
                vg[e] = self.mgu.pack(g)
                vd[e] = self.mdn.pack(dn[e])
        lib.onpu_bank_sync(self.cgu)
        lib.onpu_bank_sync(self.cdn)
        if L.last_error():
            raise L.OnpuError(L.last_error())

    def forward(self, hidden_states, indices, weights):
        lib = clib()
        h = np.ascontiguousarray(hidden_states.detach().float().cpu().numpy(), np.float32)
        ids = np.ascontiguousarray(indices.detach().cpu().numpy(), np.int32)
        w = np.ascontiguousarray(weights.detach().float().cpu().numpy(), np.float32)
        T, k = ids.shape
        y = np.empty((T, self.mdn.N), np.float32)
        if self.cffn is not None:
            ok = lib.onpu_ffn_run_many(self.cffn, L.fp(h), T, L.i32p(ids), k, L.fp(w), L.fp(y))
        else:
            lib.onpu_moe_ffn(self.cgu, self.cdn, L.fp(h), T, L.i32p(ids), k, L.fp(w), self.act_kind, self.alpha,
                             self.limit, None if self.gu_bias is None else L.fp(self.gu_bias),
                             None if self.dn_bias is None else L.fp(self.dn_bias), L.fp(y))
            ok = 1
        err = L.last_error()
        if not ok or err:
            raise L.OnpuError(err or "onpu_ffn_run_many failed")
        return torch.from_numpy(y).to(hidden_states.dtype)

    def __del__(self):
        try:
            lib = L.load()
            if getattr(self, "cffn", None):
                lib.onpu_ffn_free(self.cffn)
            else:
                for h in (getattr(self, "cgu", None), getattr(self, "cdn", None)):
                    if h:
                        lib.onpu_bank_free(h)
        except Exception:
            pass
