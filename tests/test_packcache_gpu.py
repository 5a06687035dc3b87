"""Weight blobs and the pack cache on the GPU: a matrix or expert FFN exported and imported again
gives bit-identical codes, blobs and outputs (decode GEMV, SwiGLU, two-pass, prefill GEMM, MoE
layer, and the reference's host-pointer onpu_dense_mv); the cache builds on a miss and imports
on a hit."""
import numpy as np
import pytest
import torch

from opennpu_b200 import libonpu as L
from opennpu_b200.dense import DenseMatrix, EPI_SWIGLU
from opennpu_b200.moe import ExpertFFN
from opennpu_b200.packcache import PackCache
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _x(M, K, seed):
    return torch.from_numpy(O.gen_x(M, K, seed=seed)).to(torch.bfloat16).cuda()


def _same_matrix(a, b):
    for u, v in zip(a.unpack(), b.unpack()):
        assert (u is None) == (v is None)
        if u is not None:
            assert torch.equal(u, v)
    assert np.array_equal(a.export(), b.export())


def _weights(N, K, seed):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.normal(0, 0.05, size=(N, K)).astype(np.float32)).cuda()


@pytest.mark.parametrize("kind", ["int4", "q4s", "q4nx", "gateup", "residual"])
def test_dense_round_trip_is_bit_exact(kind):
    N, K = 512, 1024
    if kind == "int4":
        v, s = O.gen_weights(N, K, seed=5)
        m = DenseMatrix.from_int4(torch.from_numpy(O.pack_baseline(v)).cuda(), torch.from_numpy(s.view(np.int16)).cuda())
    elif kind == "residual":
        m = DenseMatrix.from_float_residual(_weights(N, K, 6))
    else:
        m = DenseMatrix.from_float(_weights(N, K, 7), sym=kind != "q4nx", gateup=kind == "gateup")
    m2 = DenseMatrix.from_blob(m.export())
    assert (m2.N, m2.K, m2.fmt, m2.gateup, m2.residual) == (m.N, m.K, m.fmt, m.gateup, m.residual)
    _same_matrix(m, m2)
    for M in (1, 5, 16):
        x = _x(M, K, seed=M)
        epi = EPI_SWIGLU if kind == "gateup" else None
        assert torch.equal(m.mv(x, epi=epi), m2.mv(x, epi=epi))
    if kind in ("int4", "q4s"):
        x = _x(64, K, seed=9)
        assert torch.equal(m.mm(x), m2.mm(x))
    torch.cuda.synchronize()
    assert L.load().onpu_check_device() == 0, L.last_error()


def test_reference_upload_handle_round_trip_through_host_abi():
    N, K, sym = 256, 512, 1
    rng = np.random.default_rng(3)
    W = rng.normal(0, 0.05, size=(N, K)).astype(np.float32)
    m = DenseMatrix.from_stream(N, K, sym, O.pack(W, 8, sym))
    m2 = DenseMatrix.from_blob(m.export())
    _same_matrix(m, m2)
    lib = L.load()
    x = rng.normal(size=(3, K)).astype(np.float32)
    y1, y2 = np.empty((3, N), np.float32), np.empty((3, N), np.float32)
    fp = L.C.POINTER(L.C.c_float)
    lib.onpu_dense_mv(m.h, x.ctypes.data_as(fp), 3, y1.ctypes.data_as(fp))
    lib.onpu_dense_mv(m2.h, x.ctypes.data_as(fp), 3, y2.ctypes.data_as(fp))
    assert L.last_error() is None
    assert np.array_equal(y1, y2)


def _ffn(E=8, H=512, I=256, seed=1):
    g = torch.Generator(device="cuda").manual_seed(seed)
    gq = torch.randint(0, 256, (E, 2 * I, H // 2), dtype=torch.uint8, device="cuda", generator=g)
    gs = (torch.rand(E, 2 * I, H // 32, device="cuda", generator=g) * 0.02 + 1e-4).half()
    dq = torch.randint(0, 256, (E, H, I // 2), dtype=torch.uint8, device="cuda", generator=g)
    ds = (torch.rand(E, H, I // 32, device="cuda", generator=g) * 0.02 + 1e-4).half()
    return ExpertFFN(gq, gs, dq, ds)


def test_expert_ffn_round_trip_is_bit_exact():
    f = _ffn()
    f2 = ExpertFFN.from_blob(f.export())
    assert (f2.E, f2.H, f2.I, f2.Nd) == (f.E, f.H, f.I, f.Nd)
    assert np.array_equal(f.export(), f2.export())
    g = torch.Generator(device="cuda").manual_seed(4)
    wr = (torch.randn(f.E, f.H, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    for T in (1, 16):
        x = (torch.randn(T, f.H, device="cuda", generator=g)).to(torch.bfloat16)
        y1, ids1, w1 = f.layer(x, wr, k=2)
        y2, ids2, w2 = f2.layer(x, wr, k=2)
        assert torch.equal(ids1, ids2) and torch.equal(w1, w2) and torch.equal(y1, y2)
    torch.cuda.synchronize()
    assert L.load().onpu_check_device() == 0, L.last_error()


def test_pack_cache_builds_on_miss_and_imports_on_hit(tmp_path):
    ckpt = tmp_path / "ckpt"
    ckpt.mkdir()
    (ckpt / "model.safetensors").write_bytes(b"weights")
    W = _weights(256, 512, 11)
    built = []

    def build():
        built.append(1)
        return DenseMatrix.from_float(W)

    c = PackCache(ckpt, root=tmp_path / "cache", keep_free=0)
    a = c.dense("model.layers.0.self_attn.o_proj", build)
    assert built == [1] and c.misses == 1 and c.hits == 0
    c2 = PackCache(ckpt, root=tmp_path / "cache", keep_free=0)
    b = c2.dense("model.layers.0.self_attn.o_proj", build)
    assert built == [1] and c2.hits == 1
    x = _x(1, 512, seed=2)
    assert torch.equal(a.mv(x), b.mv(x))
    e = c2.experts("model.layers.0.mlp.experts", lambda: _ffn(E=4))
    e2 = PackCache(ckpt, root=tmp_path / "cache", keep_free=0).experts("model.layers.0.mlp.experts", None)
    assert np.array_equal(e.export(), e2.export())
    # a damaged file reads as a miss and is rebuilt and rewritten
    p = c2._path("model.layers.0.self_attn.o_proj")
    p.write_bytes(p.read_bytes()[:-64])
    c3 = PackCache(ckpt, root=tmp_path / "cache", keep_free=0)
    d = c3.dense("model.layers.0.self_attn.o_proj", build)
    assert built == [1, 1] and c3.hits == 0
    assert torch.equal(d.mv(x), a.mv(x))


def test_import_refuses_a_truncated_blob():
    m = DenseMatrix.from_float(_weights(128, 256, 12))
    b = m.export()
    with pytest.raises(L.OnpuError):
        DenseMatrix.from_blob(b[:-64])
    with pytest.raises(L.OnpuError):
        ExpertFFN.from_blob(b)                            # a dense blob is not an FFN
