"""libonpu host side, no GPU: the library loads and exports every symbol include/onpu.h declares,
and its load-time codec (geometry, search quantisers, stream-order packer, MoE CPU helpers) is
bit-exact with the oracle (itself pinned to the reference in test_oracle.py)."""
import ctypes as C
import re

import numpy as np
import pytest

from opennpu_b200 import libonpu as L
from opennpu_b200 import npu4
from oracle import oracle as O
from tests.conftest import GOLDEN, ROOT

HEADER = ROOT / "include" / "onpu.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(onpu_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = L.load()
    names = declared_functions()
    assert len(names) >= 40
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/onpu.h but not exported"
        assert n in L.SIGNATURES, f"{n} has no ctypes signature in libonpu.py"


def test_geometry_matches_reference_table():
    t = np.load(GOLDEN / "geometry.npz")["table"]
    out = (C.c_int64 * 8)()
    lib = L.load()
    for row in t:
        N, K, nc, sym = (int(v) for v in row[:4])
        lib.onpu_geometry2(N, K, nc, sym, out)
        assert tuple(out) == tuple(int(v) for v in row[4:]), (N, K, nc, sym)
        try:
            m = npu4.Mat(N, K, nc, bool(sym))
            assert (m.R, m.S, m.tiles, m.kc, m.ks, m.rows_col, m.cb, m.nbytes) == tuple(int(v) for v in row[4:])
        except ValueError:
            assert row[11] == 0


@pytest.mark.parametrize("sym", [0, 1])
@pytest.mark.parametrize("shape", [(200, 320, 8), (70, 96, 1), (130, 544, 4), (64, 2048, 1), (96, 1000, 2)])
def test_pack_and_quant_dequant_bit_exact(sym, shape):
    N, K, nc = shape
    rng = np.random.default_rng(N + K + sym)
    W = (rng.normal(0, 0.05, size=(N, K)) * rng.choice([1, 1, 10], size=(N, 1))).astype(np.float32)
    W[0, :32] = 0.0
    W[2, :32] = -0.5
    nb = O.geometry(N, K, nc, sym)[7]
    out = np.zeros(nb, np.uint8)
    assert L.load().onpu_pack(L.fp(W), N, K, nc, sym, out.ctypes.data_as(L.U8P), 3) == nb
    assert np.array_equal(out, O.pack(W, nc, sym))
    if K % 32 == 0:
        qd = np.empty_like(W)
        L.load().onpu_quant_dequant(L.fp(W), N, K, sym, L.fp(qd), 3)
        assert np.array_equal(qd, O.quant_dequant(W, sym))


def test_pack_without_geometry_returns_zero():
    W = np.zeros((5120, 17408), np.float32)[:1]     # K beyond 8 columns of 2048
    assert L.load().onpu_pack(L.fp(W), 5120, 17408, 8, 1, None, 1) == 0


def test_python_quant_sym_matches_reference_fixture():
    z = np.load(GOLDEN / "q4s.npz")
    q, d = npu4.quant_sym(z["a_W"])
    assert np.array_equal(q, z["a_q"]) and np.array_equal(d, z["a_d"])


@pytest.mark.parametrize("act", [0, 1])
def test_host_moe_act_and_sum_match_oracle(act):
    rng = np.random.default_rng(act)
    T, k, E, Ng, N = 4, 3, 6, 48, 40
    h = rng.normal(0, 2, size=(T * k, Ng)).astype(np.float32)
    ids = rng.integers(0, E, size=(T, k)).astype(np.int32)
    gb = rng.normal(0, 1, size=(E, Ng)).astype(np.float32)
    a = np.empty((T * k, Ng // 2), np.float32)
    L.load().onpu_moe_act(L.fp(h), T * k, Ng, L.i32p(ids), L.fp(gb), act, 1.702, 7.0, L.fp(a))
    a_or = np.empty_like(a)
    O.clib().or_moe_act(L.fp(h), T * k, Ng, L.i32p(ids), L.fp(gb), act, 1.702, 7.0, L.fp(a_or))
    assert np.array_equal(a, a_or)
    o = rng.normal(0, 1, size=(T * k, N)).astype(np.float32)
    w = rng.random(size=(T, k)).astype(np.float32)
    y = np.empty((T, N), np.float32)
    L.load().onpu_moe_sum(L.fp(o), T, k, N, L.i32p(ids), L.fp(w), None, L.fp(y))
    np.testing.assert_array_equal(y, O.moe_sum(o, ids, w))


def test_no_device_fails_loudly():
    lib = L.load()
    if lib.onpu_ok():
        pytest.skip("a GPU is present")
    assert lib.onpu_dense_new2(4096, 4096, 1) is None
    assert "device" in (L.last_error() or "")
    with pytest.raises(L.OnpuError):
        npu4.clib()
