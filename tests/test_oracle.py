"""Pin the CPU oracle (oracle/oracle.c + oracle/oracle.py) to the reference before trusting it.

(a) against fixtures produced by the reference's own Python (tests/golden/make_golden.py);
(b) against the reference's own libonpu host code compiled from its sources (oracle/_ref), when
    that library was built here (it needs the reference sources, so it is skipped elsewhere).
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from tests.conftest import GOLDEN


def test_geometry_matches_reference_python_mat():
    t = np.load(GOLDEN / "geometry.npz")["table"]
    for row in t:
        N, K, nc, sym = (int(v) for v in row[:4])
        assert O.geometry(N, K, nc, sym) == tuple(int(v) for v in row[4:]), (N, K, nc, sym)


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_q4nx_codec_and_stream_order(case):
    z = np.load(GOLDEN / "q4nx.npz")
    W, N, K, nc = z[f"{case}_W"], *(int(v) for v in z[f"{case}_dims"])
    q, s, m = O.requant_q4k(W)
    assert np.array_equal(q, z[f"{case}_q"])
    assert np.array_equal(s, z[f"{case}_s"]) and np.array_equal(m, z[f"{case}_m"])
    # the reference's numpy packer rounds s/m to bf16 (ml_dtypes, RNE) before writing the packets
    packed = O.pack_codes(q, O.f32_to_bf16_bits(s), O.f32_to_bf16_bits(m), nc, sym=False)
    assert np.array_equal(packed, z[f"{case}_packed"])
    q2, s2, m2 = O.unpack_codes(z[f"{case}_packed"], N, K, nc, sym=False)
    assert np.array_equal(q2, q)
    assert np.array_equal(s2, O.f32_to_bf16_bits(s)) and np.array_equal(m2, O.f32_to_bf16_bits(m))


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_q4s_codec_and_stream_order(case):
    z = np.load(GOLDEN / "q4s.npz")
    W, N, K, nc = z[f"{case}_W"], *(int(v) for v in z[f"{case}_dims"])
    q, d = O.quant_sym(W)
    assert np.array_equal(q, z[f"{case}_q"]) and np.array_equal(d, z[f"{case}_d"])
    packed = O.pack_codes(q, O.f32_to_bf16_bits(d), None, nc, sym=True, pad_code=0)   # numpy packer pads with 0
    assert np.array_equal(packed, z[f"{case}_packed"])
    q2, s2, _ = O.unpack_codes(z[f"{case}_packed"], N, K, nc, sym=True)
    assert np.array_equal(q2, q) and np.array_equal(s2, O.f32_to_bf16_bits(d))


def test_dequant_then_matmul_matches_reference_forward_path():
    z = np.load(GOLDEN / "matmul.npz")
    q, s, m = O.requant_q4k(z["W"])
    # reference.py _wq dequantises with the fp32 s/m of the min/max codec
    Wq = (q.reshape(q.shape[0], -1, 32) * s[..., None] + m[..., None]).reshape(q.shape).astype(np.float32)
    assert np.array_equal(Wq, z["Wq"])
    y = O.matmul_xwT(z["x"], Wq)
    np.testing.assert_allclose(y, z["y"], rtol=1e-5, atol=1e-5)


def test_router_matches_reference_route_with():
    z = np.load(GOLDEN / "route.npz")
    ids, w, _ = O.route(z["h"], z["Wr"], int(z["k"]))
    order = np.argsort(ids, axis=1)                  # the reference returns ids sorted ascending
    np.testing.assert_array_equal(np.take_along_axis(ids, order, 1), z["ids"])
    np.testing.assert_allclose(np.take_along_axis(w, order, 1), z["w"], rtol=1e-6)


def test_bf16_rounding_edge_cases():
    v = np.array([0.0, -0.0, 1.0, 1.00390625, 1.01171875, 3.3895314e38, np.inf, -np.inf, 1e-40], np.float32)
    b = O.f32_to_bf16_bits(v)
    assert list(b[:5]) == [0x0000, 0x8000, 0x3F80, 0x3F80, 0x3F82]   # ties to even
    assert b[6] == 0x7F80 and b[7] == 0xFF80
    nan = O.f32_to_bf16_bits(np.array([np.nan], np.float32))[0]
    assert (nan & 0x7F80) == 0x7F80 and (nan & 0x7F)


# ------------------------------------------------------------------ against the reference's C++
REF = O.ref_lib()
needs_ref = pytest.mark.skipif(REF is None, reason="oracle/_ref not built (needs the reference sources)")


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


@needs_ref
def test_geometry_matches_reference_cpp():
    t = np.load(GOLDEN / "geometry.npz")["table"]
    out = (C.c_int64 * 8)()
    for row in t:
        N, K, nc, sym = (int(v) for v in row[:4])
        REF.onpu_geometry2(N, K, nc, sym, out)
        assert tuple(out) == O.geometry(N, K, nc, sym)


@needs_ref
@pytest.mark.parametrize("sym", [0, 1])
@pytest.mark.parametrize("shape", [(200, 320, 8), (70, 96, 1), (64, 2048, 1), (130, 544, 4)])
def test_search_quantiser_and_pack_bit_exact_with_reference_cpp(sym, shape):
    N, K, nc = shape
    rng = np.random.default_rng(N * 7 + K + sym)
    W = (rng.normal(0, 0.05, size=(N, K)) * rng.choice([1, 1, 1, 10], size=(N, 1))).astype(np.float32)
    W[0, :32] = 0.0                                   # an all-zero group
    W[1, :32] = 0.25                                  # a constant group
    nb = O.geometry(N, K, nc, sym)[7]
    ref = np.zeros(nb, np.uint8)
    assert REF.onpu_pack(_fp(W), N, K, nc, sym, ref.ctypes.data_as(C.POINTER(C.c_uint8)), 2) == nb
    assert np.array_equal(O.pack(W, nc, sym), ref)
    qd_ref = np.empty_like(W)
    REF.onpu_quant_dequant(_fp(W), N, K, sym, _fp(qd_ref), 2)
    assert np.array_equal(O.quant_dequant(W, sym), qd_ref)


@needs_ref
@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("bias", [False, True])
def test_moe_act_sum_match_reference_cpp(act, bias):
    rng = np.random.default_rng(act * 2 + bias)
    T, k, E, Ng, N = 5, 4, 8, 64, 48
    h = rng.normal(0, 2, size=(T * k, Ng)).astype(np.float32)
    ids = rng.integers(0, E, size=(T, k)).astype(np.int32)
    gb = rng.normal(0, 1, size=(E, Ng)).astype(np.float32) if bias else None
    a_ref = np.empty((T * k, Ng // 2), np.float32)
    ip = ids.ctypes.data_as(C.POINTER(C.c_int32))
    REF.onpu_moe_act(_fp(h), T * k, Ng, ip, _fp(gb) if bias else None, act, 1.702, 7.0, _fp(a_ref))
    a_c = np.empty_like(a_ref)
    O.clib().or_moe_act(_fp(h), T * k, Ng, ip, _fp(gb) if bias else None, act, 1.702, 7.0, _fp(a_c))
    assert np.array_equal(a_c, a_ref)
    np.testing.assert_allclose(O.moe_act(h, ids.reshape(-1), act, 1.702, 7.0, gb), a_ref, rtol=2e-6, atol=1e-6)
    o = rng.normal(0, 1, size=(T * k, N)).astype(np.float32)
    w = rng.random(size=(T, k)).astype(np.float32)
    db = rng.normal(0, 1, size=(E, N)).astype(np.float32) if bias else None
    y_ref = np.empty((T, N), np.float32)
    REF.onpu_moe_sum(_fp(o), T, k, N, ip, _fp(w), _fp(db) if bias else None, _fp(y_ref))
    y_c = np.empty_like(y_ref)
    O.clib().or_moe_sum(_fp(o), T, k, N, ip, _fp(w), _fp(db) if bias else None, _fp(y_c))
    assert np.array_equal(y_c, y_ref)
    np.testing.assert_allclose(O.moe_sum(o, ids, w, db), y_ref, rtol=1e-6, atol=1e-6)
