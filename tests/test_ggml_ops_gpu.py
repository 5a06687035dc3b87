"""The ggml op layer on the GPU, on a small synthetic graph: a block's q/k/v weights reading one
input fuse into one stacked matrix whose first node computes all three (the others copy their
waiting slice); Q4_0, Q4_K and F32 weights; expert gate/up siblings with ids (MUL_MAT_ID); a
sibling whose input changed in between recomputes. Every output against the oracle's
dequantise-then-matmul of the weights as the layer stores them."""
import ctypes as C

import numpy as np
import pytest
import torch

from opennpu_b200 import libonpu as L
from oracle import oracle as O
from tests.test_ggml_ops import tensor
from tests.test_gguf_gpu import _oracle_codes, _oracle_weights, _rows

pytestmark = pytest.mark.gpu


def _keep(*arrays):
    return [np.ascontiguousarray(a) for a in arrays]


def _f32(shape, seed):
    return np.random.default_rng(seed).normal(0, 1, size=shape).astype(np.float32)


def _close(y, ref):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    assert np.linalg.norm(y - ref) <= 1e-5 * np.linalg.norm(ref)
    assert np.abs(y - ref).max() <= 2e-2


def test_fused_qkv_group_and_single_weights():
    lib = L.require_device()
    ctx = lib.onpu_ggml_new()
    K, M = 4096, 3
    names = [b"blk.0.attn_q.weight", b"blk.0.attn_k.weight", b"blk.0.attn_v.weight"]
    Ns = [1024, 256, 256]
    rows = [_rows(L.GGML_Q4_K, N, K, seed=10 + i) for i, N in enumerate(Ns)]
    ws = [tensor(L.GGML_Q4_K, (K, N), data=r.ctypes.data, name=nm) for r, N, nm in zip(rows, Ns, names)]
    x = _f32((M, K), 1)
    xt = tensor(L.GGML_F32, (K, M), data=x.ctypes.data, weights=0, name=b"attn_norm")
    outs = [np.zeros((M, N), np.float32) for N in Ns]
    dsts = [tensor(L.GGML_F32, (N, M), data=o.ctypes.data, weights=0, name=b"y") for o, N in zip(outs, Ns)]
    # a Q4_0 matrix and an F32 one in another block, each on its own input
    r0 = _rows(L.GGML_Q4_0, 2048, 1024, seed=20)
    w0 = tensor(L.GGML_Q4_0, (1024, 2048), data=r0.ctypes.data, name=b"blk.1.ffn_down.weight")
    Wf = (_f32((1024, 1024), 21) * 0.05).astype(np.float32)
    wf = tensor(L.GGML_F32, (1024, 1024), data=Wf.ctypes.data, name=b"blk.1.attn_output.weight")
    x0, xf = _f32((2, 1024), 2), _f32((1, 1024), 3)
    x0t = tensor(L.GGML_F32, (1024, 2), data=x0.ctypes.data, weights=0, name=b"a")
    xft = tensor(L.GGML_F32, (1024, 1), data=xf.ctypes.data, weights=0, name=b"b")
    y0, yf = np.zeros((2, 2048), np.float32), np.zeros((1, 1024), np.float32)
    d0 = tensor(L.GGML_F32, (2048, 2), data=y0.ctypes.data, weights=0, name=b"y0")
    df = tensor(L.GGML_F32, (1024, 1), data=yf.ctypes.data, weights=0, name=b"yf")
    for w, xx in list(zip(ws, [xt] * 3)) + [(w0, x0t), (wf, xft)]:
        lib.onpu_ggml_note(ctx, L.GGML_OP_MUL_MAT, C.byref(w), C.byref(xx), None)
    for w, d in zip(ws, dsts):
        assert lib.onpu_ggml_compute(ctx, L.GGML_OP_MUL_MAT, C.byref(d), C.byref(w), C.byref(xt), None) == 0, \
            L.last_error()
    assert lib.onpu_ggml_compute(ctx, L.GGML_OP_MUL_MAT, C.byref(d0), C.byref(w0), C.byref(x0t), None) == 0
    assert lib.onpu_ggml_compute(ctx, L.GGML_OP_MUL_MAT, C.byref(df), C.byref(wf), C.byref(xft), None) == 0
    st = (C.c_int64 * 4)()
    lib.onpu_ggml_stats(ctx, st)
    assert list(st) == [2, 0, 1, 3]                  # k and v from the fused call; 1 group; 3 handles
    for r, N, o in zip(rows, Ns, outs):
        _close(o, O.matmul_xwT(x, _oracle_weights(L.GGML_Q4_K, *_oracle_codes(L.GGML_Q4_K, r, N, K))))
    _close(y0, O.matmul_xwT(x0, _oracle_weights(L.GGML_Q4_0, *_oracle_codes(L.GGML_Q4_0, r0, 2048, 1024))))
    _close(yf, O.matmul_xwT(xf, O.quant_dequant(Wf, 0)))     # q4nx search quantiser, as the reference
    # a sibling whose input changed between the leader and its own node: recomputed on its own
    assert lib.onpu_ggml_compute(ctx, L.GGML_OP_MUL_MAT, C.byref(dsts[0]), C.byref(ws[0]), C.byref(xt), None) == 0
    x[:] = _f32((M, K), 5)
    assert lib.onpu_ggml_compute(ctx, L.GGML_OP_MUL_MAT, C.byref(dsts[1]), C.byref(ws[1]), C.byref(xt), None) == 0
    lib.onpu_ggml_stats(ctx, st)
    assert st[1] == 1
    _close(outs[1], O.matmul_xwT(x, _oracle_weights(L.GGML_Q4_K, *_oracle_codes(L.GGML_Q4_K, rows[1], Ns[1], K))))
    lib.onpu_ggml_free(ctx)


@pytest.mark.parametrize("type_", [L.GGML_Q4_K, L.GGML_Q4_0])
def test_fused_expert_gate_up(type_):
    lib = L.require_device()
    ctx = lib.onpu_ggml_new()
    E, N, K, T, k = 8, 256, 512, 4, 2
    rg, ru = _rows(type_, E * N, K, seed=30), _rows(type_, E * N, K, seed=31)
    wg = tensor(type_, (K, N, E), data=rg.ctypes.data, name=b"blk.2.ffn_gate_exps.weight")
    wu = tensor(type_, (K, N, E), data=ru.ctypes.data, name=b"blk.2.ffn_up_exps.weight")
    x = _f32((T, K), 6)
    xt = tensor(L.GGML_F32, (K, 1, T), data=x.ctypes.data, weights=0, name=b"ffn_norm")
    rng = np.random.default_rng(7)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    idt = tensor(L.GGML_I32, (k, T), data=ids.ctypes.data, weights=0, name=b"ids")
    yg, yu = np.zeros((T, k, N), np.float32), np.zeros((T, k, N), np.float32)
    dg = tensor(L.GGML_F32, (N, k, T), data=yg.ctypes.data, weights=0, name=b"g")
    du = tensor(L.GGML_F32, (N, k, T), data=yu.ctypes.data, weights=0, name=b"u")
    for w in (wg, wu):
        lib.onpu_ggml_note(ctx, L.GGML_OP_MUL_MAT_ID, C.byref(w), C.byref(xt), C.byref(idt))
    assert lib.onpu_ggml_compute(ctx, L.GGML_OP_MUL_MAT_ID, C.byref(dg), C.byref(wg), C.byref(xt), C.byref(idt)) == 0, \
        L.last_error()
    assert lib.onpu_ggml_compute(ctx, L.GGML_OP_MUL_MAT_ID, C.byref(du), C.byref(wu), C.byref(xt), C.byref(idt)) == 0
    st = (C.c_int64 * 4)()
    lib.onpu_ggml_stats(ctx, st)
    assert st[0] == 1 and st[2] == 1
    for rr, y in ((rg, yg), (ru, yu)):
        W = _oracle_weights(type_, *_oracle_codes(type_, rr, E * N, K)).reshape(E, N, K)
        for t in range(T):
            for j in range(k):
                _close(y[t, j], O.matmul_xwT(x[t][None], W[ids[t, j]])[0])
    lib.onpu_ggml_free(ctx)
