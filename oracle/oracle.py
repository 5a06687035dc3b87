"""ORACLE — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / ``--impl reference`` legs may
import this module, and only as the checker or as the timed CPU baseline. The product
(``opennpu_b200`` and its libonpu.so) never imports, links or calls it.

A numpy restatement of the reference's CPU path for int4 group-32 weight-only matmul, plus a
ctypes loader for the plain-C restatement in ``oracle.c`` (quantisers, geometry, stream-order
packer). Reference lines followed (paths relative to the reference project root):

- ``requant_q4k``      opennpu/native/runtime.py:74-82 (min/max per-32 affine codec)
- ``quant_sym``        opennpu/native/npu4/model.py:127-147 (numpy q4s quantiser, 5 candidates)
- ``dequant``          opennpu/native/reference.py:24-28 (q*s + m), onpu_api.cpp:517-518 ((q-8)*d)
- ``matmul_xwT``       opennpu/native/reference.py:55-57 (h @ W.T, fp32 torch on the host)
- ``route``            opennpu/native/reference.py:71-76 (softmax -> topk -> renormalise)
- ``moe_ffn``          opennpu/native/reference.py:77-84 (per-expert SwiGLU, weighted sum)
- ``moe_act/moe_sum``  llama/ggml-opennpu/onpu_cpu.cpp:233-274
- ``attn_step``        llama/ggml-opennpu/onpu_cpu.cpp:173-218 (decode attention, GQA, mask, sinks)
- ``q4k_transcode``    llama/ggml-opennpu/ggml-opennpu.cpp:100-143 (GGUF Q4_K -> q4nx codes, bf16 s / m)
- ``q4_0_codes``       the GGUF Q4_0 block (the ggml format the reference reads through to_float,
                       ggml-opennpu.cpp:77-86) unpacked: codes and fp16 scale

Parity pin: tests/test_oracle.py checks these against the reference's own code — its Python
imported in the container that generated tests/golden/*.npz (tests/golden/make_golden.py) and its
C++ host code compiled into oracle/_ref (oracle/Makefile ``ref``).
"""
import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
REF_LIB = HERE / "_ref" / "libonpu_ref.so"

# weight formats (the codes are always q in 0..15)
FMT_Q4NX = 0      # w = q * s + m, bf16 s/m                (reference default "q4nx")
FMT_Q4S = 1       # w = (q - 8) * d, bf16 d                 (reference "q4s")
FMT_Q4F16 = 2     # w = (q - 8) * s = v * s, fp16 s          (BASELINE layout: v in [-8, 7])

GROUP = 32


# ------------------------------------------------------------------ 16-bit floats
def f32_to_bf16_bits(a):
    """fp32 -> bf16 bits, round to nearest even; NaN keeps its top bits with the quiet bit set
    (opennpu_core.hpp:50-56)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, ((u >> 16) | 64) & 0xFFFF, r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b):
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(a):
    """fp32 values rounded to the nearest bf16 value (returned as fp32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(a))


def f16_bits_to_f32(b):
    return np.asarray(b, np.uint16).view(np.float16).astype(np.float32)


# ------------------------------------------------------------------ synthetic BASELINE inputs
def gen_weights(N, K, seed=0):
    """BASELINE weights: v ~ U{-8..7} int, fp16 scales |N(0, 0.02)| + 1e-4 per 32 along K.
    One default_rng(seed) stream, tensors drawn in a fixed order (v, then s)."""
    assert K % GROUP == 0
    rng = np.random.default_rng(seed)
    v = rng.integers(-8, 8, size=(N, K), dtype=np.int8)
    s = (np.abs(rng.normal(0.0, 0.02, size=(N, K // GROUP))) + 1e-4).astype(np.float16)
    return v, s


def gen_x(M, K, seed=0):
    """Activations: N(0, 1) rounded to bf16 (returned as fp32 holding bf16 values)."""
    rng = np.random.default_rng(seed)
    return round_bf16(rng.normal(0.0, 1.0, size=(M, K)).astype(np.float32))


def pack_baseline(v):
    """BASELINE packing: int4 two's complement, 2 per byte along K, element 2j in the low nibble
    of byte j. v [N][K] int8 in [-8, 7] -> uint8 [N][K/2]."""
    u = (np.asarray(v, np.int16) & 0xF).astype(np.uint8)
    return (u[:, 0::2] | (u[:, 1::2] << 4)).astype(np.uint8)


def unpack_baseline(p, K):
    p = np.asarray(p, np.uint8)
    lo = (p & 0xF).astype(np.int8)
    hi = (p >> 4).astype(np.int8)
    v = np.empty((p.shape[0], K), np.int8)
    v[:, 0::2] = np.where(lo > 7, lo - 16, lo)
    v[:, 1::2] = np.where(hi > 7, hi - 16, hi)
    return v


# ------------------------------------------------------------------ codecs
def requant_q4k(W, group=GROUP):
    """runtime.py:74-82: per-32 affine 4-bit, w ~= q*scale + min, min/max grid (fp32 s/m)."""
    M_, K = W.shape
    Wg = W.reshape(M_, K // group, group)
    mn = Wg.min(2)
    sc = (Wg.max(2) - mn) / 15.0
    sc = np.where(sc <= 0, 1.0, sc).astype(np.float32)
    q = np.clip(np.rint((Wg - mn[..., None]) / sc[..., None]), 0, 15).astype(np.uint8)
    return q.reshape(M_, K), sc, mn.astype(np.float32)


def quant_sym(W, group=GROUP):
    """model.py:127-147: q4s with 5 candidate scales around absmax/8, bf16-exact d (values)."""
    M_, K = W.shape
    g = W.reshape(M_, K // group, group)
    mx = np.take_along_axis(g, np.abs(g).argmax(2)[..., None], 2)[..., 0]
    best_q = best_d = best_e = None
    for div in (-8.0, -7.5, -7.0, 7.0, 7.5):
        d = round_bf16(np.asarray(mx / div, np.float32))
        d = np.where(d == 0, 1.0, d).astype(np.float32)
        q = np.clip(np.rint(g / d[..., None]), -8, 7)
        e = ((q * d[..., None] - g) ** 2).sum(2)
        if best_e is None:
            best_q, best_d, best_e = q, d, e
        else:
            m = e < best_e
            best_q = np.where(m[..., None], q, best_q)
            best_d = np.where(m, d, best_d)
            best_e = np.minimum(e, best_e)
    return (best_q + 8).astype(np.uint8).reshape(M_, K), best_d


def dequant(q, s_bits, m_bits, fmt):
    """Codes -> fp32 W (reference.py:24-28; onpu_api.cpp:517-518). q [N][K] uint8 0..15;
    s_bits/m_bits [N][K/32] uint16 (bf16 or fp16 bits by fmt)."""
    q = np.asarray(q, np.float32)
    N, K = q.shape
    qg = q.reshape(N, K // GROUP, GROUP)
    if fmt == FMT_Q4NX:
        W = qg * bf16_bits_to_f32(s_bits)[..., None] + bf16_bits_to_f32(m_bits)[..., None]
    elif fmt == FMT_Q4S:
        W = (qg - 8.0) * bf16_bits_to_f32(s_bits)[..., None]
    else:
        W = (qg - 8.0) * f16_bits_to_f32(s_bits)[..., None]
    return W.reshape(N, K).astype(np.float32)


def dequant_baseline(v, s):
    """BASELINE (v int8 [-8,7], s fp16) -> fp32 W = v * s."""
    N, K = v.shape
    return (v.reshape(N, K // GROUP, GROUP).astype(np.float32)
            * np.asarray(s, np.float16).astype(np.float32)[..., None]).reshape(N, K)


def matmul_xwT(x, W, acc=np.float64):
    """y = x @ W.T (reference.py:55-57). The oracle accumulates in float64 by default."""
    return (np.asarray(x, acc) @ np.asarray(W, acc).T).astype(np.float32)


# ------------------------------------------------------------------ MoE (reference.py:71-84)
def route(h, Wr, k, norm_topk_prob=True):
    """softmax(h @ Wr.T) -> top-k (descending probability, lower expert id first on ties) ->
    renormalise. h [T][H] fp32, Wr [E][H] fp32. Returns ids int32 [T][k], w fp32 [T][k]."""
    logits = np.asarray(h, np.float64) @ np.asarray(Wr, np.float64).T
    z = logits - logits.max(-1, keepdims=True)
    e = np.exp(z)
    prob = e / e.sum(-1, keepdims=True)
    order = np.argsort(-prob, axis=-1, kind="stable")[:, :k]
    w = np.take_along_axis(prob, order, -1)
    if norm_topk_prob:
        w = w / w.sum(-1, keepdims=True)
    return order.astype(np.int32), w.astype(np.float32), logits.astype(np.float32)


def silu(a):
    a = np.asarray(a, np.float64)
    return a / (1.0 + np.exp(-a))


def moe_ffn(h, ids, w, Wg, Wu, Wd):
    """reference.py:77-84: for each token t and slot j (expert e = ids[t, j]),
    y_t += w[t, j] * (silu(h_t Wg_e^T) * (h_t Wu_e^T)) Wd_e^T. Wg/Wu/Wd: callables e -> fp32
    matrices (gate [I][H], up [I][H], down [H][I]). Accumulates in float64; the activation between
    the projections is not rounded (the reference computes it in fp32)."""
    T = h.shape[0]
    out = np.zeros((T, Wd(int(ids[0, 0])).shape[0]), np.float64)
    for e in np.unique(ids):
        rows, slots = np.nonzero(ids == e)
        hh = np.asarray(h[rows], np.float64)
        a = silu(hh @ np.asarray(Wg(int(e)), np.float64).T) * (hh @ np.asarray(Wu(int(e)), np.float64).T)
        o = a @ np.asarray(Wd(int(e)), np.float64).T
        out[rows] += w[rows, slots][:, None] * o
    return out.astype(np.float32)


def moe_act(h, ids, act=0, alpha=1.702, limit=7.0, gu_bias=None):
    """onpu_cpu.cpp:233-256 (numpy)."""
    h = np.asarray(h, np.float32)
    if gu_bias is not None:
        h = h + np.asarray(gu_bias, np.float32)[ids]
    Ng = h.shape[-1]
    I = Ng // 2
    if act == 1:
        g = np.minimum(h[:, 0::2], limit)
        u = np.clip(h[:, 1::2], -limit, limit)
        return ((u + 1.0) * g / (1.0 + np.exp(-alpha * g))).astype(np.float32)
    return (h[:, :I] / (1.0 + np.exp(-h[:, :I])) * h[:, I:]).astype(np.float32)


def moe_sum(o, ids, w, bias=None):
    """onpu_cpu.cpp:259-274 (numpy): y[t] = sum_j w[t,j] * (o[t,j] + bias[ids[t,j]])."""
    o = np.asarray(o, np.float32)
    T, k = ids.shape
    if bias is not None:
        o = o + np.asarray(bias, np.float32)[ids.reshape(-1)].reshape(o.shape)
    return (o.reshape(T, k, -1) * w[:, :, None]).sum(1).astype(np.float32)


# ------------------------------------------------------------------ GGUF blocks
def q4_0_codes(blocks):
    """GGUF Q4_0 blocks uint8 [nb, 18] -> codes uint8 [nb, 32] (w = (q - 8) * d) and the fp16 d bits
    uint16 [nb]: byte j holds element j (low nibble) and element j + 16 (high nibble)."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 18)
    d = b[:, :2].copy().view(np.uint16)[:, 0]
    qs = b[:, 2:]
    return np.concatenate([qs & 15, qs >> 4], axis=1).astype(np.uint8), d


def q4k_scale_min(sc, sub):
    """6-bit scale and min of sub-block `sub` (0..7) from the 12 packed bytes sc [..., 12]."""
    sc = sc.astype(np.int32)
    if sub < 4:
        return sc[..., sub] & 63, sc[..., sub + 4] & 63
    return ((sc[..., sub + 4] & 0xF) | ((sc[..., sub - 4] >> 6) << 4),
            (sc[..., sub + 4] >> 4) | ((sc[..., sub] >> 6) << 4))


def _bf_step(h, direction):
    """The bf16 value next to h (bits, uint16 array) upwards (+1) or downwards (-1) in value; from
    zero, the smallest subnormal of that sign (ggml-opennpu.cpp:106-110)."""
    f = bf16_bits_to_f32(h)
    step = np.where((f > 0) == (direction > 0), h.astype(np.int32) + 1, h.astype(np.int32) - 1)
    zero = np.uint16(0x0001 if direction > 0 else 0x8001)
    return np.where(f == 0, zero, step.astype(np.uint16)).astype(np.uint16)


def q4k_transcode(blocks):
    """GGUF Q4_K super-blocks uint8 [nb, 144] -> q4nx: codes uint8 [nb, 8, 32], bf16 scale and min
    bits uint16 [nb, 8], as ggml-opennpu.cpp:114-143 (q4k_codes): the codes of sub-block b, exact
    weights q * S + M with S = d * sc_b and M = -dmin * m_b (fp32), then among the 3 x 3 bf16 pairs
    next to (bf16(S), bf16(M)) the first (in ds-major order) with the least fp32 sum of squared
    errors, every float operation rounded separately in the reference's order."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 144)
    nb = b.shape[0]
    d = b[:, 0:2].copy().view(np.float16)[:, 0].astype(np.float32)
    dmin = b[:, 2:4].copy().view(np.float16)[:, 0].astype(np.float32)
    sc, qs = b[:, 4:16], b[:, 16:144]
    q = np.empty((nb, 8, 32), np.uint8)
    s_out = np.empty((nb, 8), np.uint16)
    m_out = np.empty((nb, 8), np.uint16)
    for sub in range(8):
        sv, mv = q4k_scale_min(sc, sub)
        qq = qs[:, (sub // 2) * 32:(sub // 2) * 32 + 32]
        q[:, sub] = (qq >> 4) if sub & 1 else (qq & 15)
        qf = q[:, sub].astype(np.float32)
        S = (d * sv.astype(np.float32)).astype(np.float32)
        M = ((-dmin) * mv.astype(np.float32)).astype(np.float32)
        s0, m0 = f32_to_bf16_bits(S), f32_to_bf16_bits(M)
        best = np.full(nb, np.inf, np.float32)
        bs, bm = s0.copy(), m0.copy()
        for ds in (-1, 0, 1):
            for dm in (-1, 0, 1):
                sc_ = _bf_step(s0, ds) if ds else s0
                mn_ = _bf_step(m0, dm) if dm else m0
                sf, mf = bf16_bits_to_f32(sc_), bf16_bits_to_f32(mn_)
                e = np.zeros(nb, np.float32)
                for l in range(32):
                    x = ((qf[:, l] * sf) + mf) - ((qf[:, l] * S) + M)
                    e = e + x * x
                take = e < best
                best = np.where(take, e, best)
                bs = np.where(take, sc_, bs)
                bm = np.where(take, mn_, bm)
        s_out[:, sub], m_out[:, sub] = bs, bm
    return q, s_out, m_out


def q4k_exact(blocks):
    """The exact fp32 weights of Q4_K super-blocks [nb, 144] -> [nb, 256]: q * (d * sc) - dmin * m."""
    b = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 144)
    d = b[:, 0:2].copy().view(np.float16)[:, 0].astype(np.float32)
    dmin = b[:, 2:4].copy().view(np.float16)[:, 0].astype(np.float32)
    out = np.empty((b.shape[0], 8, 32), np.float32)
    for sub in range(8):
        sv, mv = q4k_scale_min(b[:, 4:16], sub)
        qq = b[:, 16 + (sub // 2) * 32:16 + (sub // 2) * 32 + 32]
        qf = ((qq >> 4) if sub & 1 else (qq & 15)).astype(np.float32)
        S = (d * sv.astype(np.float32)).astype(np.float32)
        dm = (dmin * mv.astype(np.float32)).astype(np.float32)
        out[:, sub] = qf * S[:, None] - dm[:, None]
    return out.reshape(-1, 256)


# ------------------------------------------------------------------ the C restatement
_LIB = None


def build_c():
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)


def clib():
    """ctypes handle on oracle.c (built on first use if missing)."""
    global _LIB
    if _LIB is None:
        if not LIB.exists():
            build_c()
        L = C.CDLL(str(LIB))
        I64, U8P, U16P, FP = C.c_int64, C.POINTER(C.c_uint8), C.POINTER(C.c_uint16), C.POINTER(C.c_float)
        L.or_geometry.argtypes = [I64, I64, C.c_int, C.c_int, C.POINTER(I64)]
        L.or_pack.restype = I64
        L.or_pack.argtypes = [FP, I64, I64, C.c_int, C.c_int, U8P]
        L.or_pack_codes.restype = I64
        L.or_pack_codes.argtypes = [U8P, U16P, U16P, I64, I64, C.c_int, C.c_int, C.c_int, U8P]
        L.or_unpack_codes.restype = I64
        L.or_unpack_codes.argtypes = [U8P, I64, I64, C.c_int, C.c_int, U8P, U16P, U16P]
        L.or_quant_dequant.argtypes = [FP, I64, I64, C.c_int, FP]
        L.or_quant_sym32.argtypes = [FP, U8P, U16P]
        L.or_quant_asym32.argtypes = [FP, U8P, U16P, U16P]
        L.or_moe_act.argtypes = [FP, I64, I64, C.POINTER(C.c_int32), FP, C.c_int, C.c_float, C.c_float, FP]
        L.or_moe_sum.argtypes = [FP, I64, C.c_int, I64, C.POINTER(C.c_int32), FP, FP, FP]
        _LIB = L
    return _LIB


def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t))


def geometry(N, K, ncols, sym):
    out = (C.c_int64 * 8)()
    clib().or_geometry(N, K, ncols, int(sym), out)
    return tuple(out)


def pack(W, ncols, sym):
    W = np.ascontiguousarray(W, np.float32)
    N, K = W.shape
    nb = geometry(N, K, ncols, sym)[7]
    out = np.zeros(nb, np.uint8)
    if nb:
        clib().or_pack(_p(W, C.c_float), N, K, ncols, int(sym), _p(out, C.c_uint8))
    return out


def pack_codes(q, s, m, ncols, sym, pad_code=-1):
    """Codes -> stream order. pad_code -1: the C++ packer's padding (8 for q4s, else 0); 0: the
    numpy packer's."""
    q = np.ascontiguousarray(q, np.uint8)
    N, K = q.shape
    s = np.ascontiguousarray(s, np.uint16)
    m = np.ascontiguousarray(m if m is not None else np.zeros_like(s), np.uint16)
    nb = geometry(N, K, ncols, sym)[7]
    out = np.zeros(nb, np.uint8)
    if nb:
        clib().or_pack_codes(_p(q, C.c_uint8), _p(s, C.c_uint16), _p(m, C.c_uint16), N, K, ncols, int(sym),
                             int(pad_code), _p(out, C.c_uint8))
    return out


def unpack_codes(buf, N, K, ncols, sym):
    buf = np.ascontiguousarray(buf, np.uint8)
    q = np.zeros((N, K), np.uint8)
    s = np.zeros((N, K // GROUP), np.uint16)
    m = np.zeros((N, K // GROUP), np.uint16)
    clib().or_unpack_codes(_p(buf, C.c_uint8), N, K, ncols, int(sym), _p(q, C.c_uint8), _p(s, C.c_uint16),
                           _p(m, C.c_uint16))
    return q, s, (None if sym else m)


def quant_dequant(W, sym):
    W = np.ascontiguousarray(W, np.float32)
    out = np.empty_like(W)
    clib().or_quant_dequant(_p(W, C.c_float), W.shape[0], W.shape[1], int(sym), _p(out, C.c_float))
    return out


def quantize_codes(W, sym):
    """The search quantisers (opennpu_core.hpp:103-169) per 32 -> (q, s_bits, m_bits|None)."""
    W = np.ascontiguousarray(W, np.float32)
    N, K = W.shape
    q = np.zeros((N, K), np.uint8)
    s = np.zeros((N, K // GROUP), np.uint16)
    m = np.zeros((N, K // GROUP), np.uint16)
    L = clib()
    for r in range(N):
        for g in range(K // GROUP):
            xg = np.ascontiguousarray(W[r, g * GROUP:(g + 1) * GROUP])
            qg = np.zeros(GROUP, np.uint8)
            sb, mb = C.c_uint16(), C.c_uint16()
            if sym:
                L.or_quant_sym32(_p(xg, C.c_float), _p(qg, C.c_uint8), C.byref(sb))
            else:
                L.or_quant_asym32(_p(xg, C.c_float), _p(qg, C.c_uint8), C.byref(sb), C.byref(mb))
            q[r, g * GROUP:(g + 1) * GROUP] = qg
            s[r, g], m[r, g] = sb.value, mb.value
    return q, s, (None if sym else m)


def ref_lib():
    """The reference's own libonpu host code (oracle/_ref), or None when it was not built here."""
    if not REF_LIB.exists():
        return None
    os.environ.setdefault("OPENNPU_GEMV_DIR", "/nonexistent-opennpu-gemv")
    os.environ.setdefault("OPENNPU_GEMM8_DIR", "/nonexistent-opennpu-gemm8")
    L = C.CDLL(str(REF_LIB))
    I64, FP = C.c_int64, C.POINTER(C.c_float)
    L.onpu_geometry2.argtypes = [I64, I64, C.c_int, C.c_int, C.POINTER(I64)]
    L.onpu_pack.restype = I64
    L.onpu_pack.argtypes = [FP, I64, I64, C.c_int, C.c_int, C.POINTER(C.c_uint8), C.c_int]
    L.onpu_quant_dequant.argtypes = [FP, I64, I64, C.c_int, FP, C.c_int]
    L.onpu_moe_act.argtypes = [FP, I64, I64, C.POINTER(C.c_int32), FP, C.c_int, C.c_float, C.c_float, FP]
    L.onpu_moe_sum.argtypes = [FP, I64, C.c_int, I64, C.POINTER(C.c_int32), FP, FP, FP]
    at = [FP, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_int, I64, I64, I64, FP, FP, C.c_float, FP]
    L.onpu_attn_step.argtypes = at
    L.onpu_attn_step_bf16.argtypes = at
    return L


# ------------------------------------------------------------------ decode attention
def attn_step(q, K, V, mask=None, sinks=None, scale=None):
    """One decode token of softmax attention, llama/ggml-opennpu/onpu_cpu.cpp:185-218, in float64
    (a truth for the GPU's fp32 sums). q [Hq, D]; K, V [Hkv, S, D] (fp32 values; a bf16 cache is
    passed widened); mask [S] additive; sinks [Hq]: an extra logit per head that takes probability
    mass and has no value. Query head h reads kv head h // (Hq // Hkv). S = 0 gives zeros; every
    score -inf with no sink gives NaN, as the reference's exp(-inf - -inf)."""
    q = np.asarray(q, np.float64)
    K = np.asarray(K, np.float64)
    V = np.asarray(V, np.float64)
    Hq, D = q.shape
    Hkv, S, _ = K.shape
    rep = Hq // Hkv
    scale = D ** -0.5 if scale is None else scale
    out = np.zeros((Hq, D), np.float64)
    with np.errstate(invalid="ignore", over="ignore"):
        for h in range(Hq):
            s = (K[h // rep] @ q[h]) * scale
            if mask is not None:
                s = s + np.asarray(mask, np.float64)
            mx = max([float(sinks[h])] if sinks is not None else [-np.inf])
            if S:
                mx = max(mx, float(s.max()))
            p = np.exp(s - mx)
            tot = p.sum() + (np.exp(float(sinks[h]) - mx) if sinks is not None else 0.0)
            if S:
                out[h] = (p / tot) @ V[h // rep]
    return out


def attn_step_ref(L, q, K, V, mask=None, sinks=None, scale=None, bf16=False):
    """The reference's own onpu_attn_step(_bf16) from oracle/_ref on contiguous [Hkv, S, D] arrays
    (K, V float32, or uint16 bf16 bits with bf16=True)."""
    q = np.ascontiguousarray(q, np.float32)
    K = np.ascontiguousarray(K)
    V = np.ascontiguousarray(V)
    Hq, D = q.shape
    Hkv, S, _ = K.shape
    out = np.zeros((Hq, D), np.float32)
    fp = lambda a: None if a is None else np.ascontiguousarray(a, np.float32).ctypes.data_as(C.POINTER(C.c_float))
    m = None if mask is None else np.ascontiguousarray(mask, np.float32)
    sk = None if sinks is None else np.ascontiguousarray(sinks, np.float32)
    f = L.onpu_attn_step_bf16 if bf16 else L.onpu_attn_step
    f(fp(q), Hq, D, K.ctypes.data, V.ctypes.data, Hkv, S, S * D, D, fp(m), fp(sk),
      float(D ** -0.5 if scale is None else scale), fp(out))
    return out
