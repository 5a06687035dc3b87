"""GPU parity of the grouped expert GEMV (onpu_bank_run), the routed-expert FFN (onpu_moe_ffn,
onpu_ffn_run / run_many) and the reference engine's NPUExperts call shape, against the oracle."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from opennpu_b200 import libonpu as L
    return L


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def make_bank(L, E, N, K, sym, seed, ncols=1):
    rng = np.random.default_rng(seed)
    Ws = rng.normal(0, 0.05, size=(E, N, K)).astype(np.float32)
    lib = L.load()
    h = lib.onpu_bank_new2(N, K, E, ncols, sym)
    assert h, L.last_error()
    nb = lib.onpu_bank_expert_bytes(h)
    buf = np.ctypeslib.as_array(lib.onpu_bank_buf(h), shape=(E, nb))
    deq = []
    for e in range(E):
        buf[e] = O.pack(Ws[e], ncols, sym)
        q, s, m = O.unpack_codes(buf[e], N, K, ncols, sym)
        deq.append(O.dequant(q, s, m, O.FMT_Q4S if sym else O.FMT_Q4NX))
    lib.onpu_bank_sync(h)
    assert L.last_error() is None
    return h, np.stack(deq)


@pytest.mark.parametrize("sym", [0, 1])
@pytest.mark.parametrize("T,k,x_per_slot", [(1, 8, 0), (5, 2, 0), (20, 8, 0), (7, 4, 1), (40, 1, 0)])
def test_bank_run_matches_oracle(sym, T, k, x_per_slot):
    L = _lib()
    E, N, K = 12, 192, 256
    h, Wd = make_bank(L, E, N, K, sym, seed=T * 10 + k)
    rng = np.random.default_rng(T)
    ids = rng.integers(0, E, size=(T, k)).astype(np.int32)
    ids[0, :] = 3                                   # a hot expert (more than 16 slots when T large)
    xr = T * k if x_per_slot else T
    x = np.ascontiguousarray(rng.normal(0, 1, size=(xr, K)).astype(np.float32))
    y = np.empty((T, k, N), np.float32)
    L.load().onpu_bank_run(h, L.fp(x), x_per_slot, T, L.i32p(ids), k, L.fp(y))
    assert L.last_error() is None
    xb = x                                          # K = 256: fp32 inputs staged exactly (two fp16 halves)
    for t in range(T):
        for j in range(k):
            xin = xb[t * k + j] if x_per_slot else xb[t]
            ref = O.matmul_xwT(xin[None], Wd[ids[t, j]])[0]
            assert rel_l2(y[t, j], ref) < 1e-5
    L.load().onpu_bank_free(h)


def test_bank_run_rejects_bad_expert_id():
    L = _lib()
    h, _ = make_bank(L, 4, 64, 64, 1, seed=0)
    ids = np.array([[0, 4]], np.int32)
    x = np.zeros((1, 64), np.float32)
    y = np.zeros((1, 2, 64), np.float32)
    L.load().onpu_bank_run(h, L.fp(x), 0, 1, L.i32p(ids), 2, L.fp(y))
    assert "out of range" in (L.last_error() or "")
    L.load().onpu_bank_free(h)


def moe_reference(x, ids, w, Wg, Wd, act=0, alpha=1.702, limit=7.0, gb=None, db=None):
    """reference.py:77-84 / onpu_moe_ffn semantics (onpu_cpu.cpp:233-274 for the activation and
    the weighted sum) on dequantised weights: fp32 activations throughout, float64 sums."""
    T, k = ids.shape
    hrows = np.stack([O.matmul_xwT(x[t][None], Wg[ids[t, j]])[0] for t in range(T) for j in range(k)])
    a = O.moe_act(hrows, ids.reshape(-1), act, alpha, limit, gb)
    o = np.stack([O.matmul_xwT(a[t * k + j][None], Wd[ids[t, j]])[0] for t in range(T) for j in range(k)])
    return O.moe_sum(o, ids, w, db)


def assert_close(y, ref):
    """The north-star bound: rel-L2 <= 1e-3 and max-abs <= 2e-2 against the fp32 oracle."""
    y = np.asarray(y, np.float64)
    assert np.isfinite(y).all()
    assert rel_l2(y, ref) <= 1e-3, rel_l2(y, ref)
    assert np.abs(y - ref).max() <= 2e-2, np.abs(y - ref).max()


@pytest.mark.parametrize("act,bias", [(0, False), (0, True), (1, True)])
@pytest.mark.parametrize("T", [1, 16])
def test_moe_ffn_matches_oracle(act, bias, T):
    L = _lib()
    E, H, I, k = 8, 256, 128, 4
    gu, Wg = make_bank(L, E, 2 * I, H, 1, seed=1)
    dn, Wd = make_bank(L, E, H, I, 1, seed=2)
    rng = np.random.default_rng(T + act)
    x = O.round_bf16(rng.normal(0, 1, size=(T, H)).astype(np.float32))      # bf16 activations (BASELINE)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    w = rng.random(size=(T, k)).astype(np.float32)
    gb = rng.normal(0, 0.1, size=(E, 2 * I)).astype(np.float32) if bias else None
    db = rng.normal(0, 0.1, size=(E, H)).astype(np.float32) if bias else None
    y = np.empty((T, H), np.float32)
    L.load().onpu_moe_ffn(gu, dn, L.fp(x), T, L.i32p(ids), k, L.fp(w), act, 1.702, 7.0,
                          None if gb is None else L.fp(gb), None if db is None else L.fp(db), L.fp(y))
    assert L.last_error() is None
    ref = moe_reference(x, ids, w, Wg, Wd, act, 1.702, 7.0, gb, db)
    assert_close(y, ref)
    L.load().onpu_bank_free(gu)
    L.load().onpu_bank_free(dn)


@pytest.mark.parametrize("T", [1, 3, 64])
def test_fused_ffn_and_npu_experts(T):
    _lib()
    from opennpu_b200 import npu4
    E, H, I, k = 16, 256, 128, 8
    rng = np.random.default_rng(T)
    gu = rng.normal(0, 0.05, size=(E, 2 * I, H)).astype(np.float32)
    dn = rng.normal(0, 0.05, size=(E, H, I)).astype(np.float32)
    ex = npu4.NPUExperts(list(gu), list(dn), topk=k, sym=True)
    assert ex.cffn is not None                          # gate_up + down fused path
    x = torch.randn(T, H).bfloat16().float()           # bf16 activations (BASELINE)
    idx = torch.stack([torch.randperm(E)[:k] for _ in range(T)])
    wts = torch.rand(T, k)
    y = ex(x, idx, wts).numpy()
    Wg = np.stack([npu4.quant_dequant(gu[e], sym=True) for e in range(E)])
    Wd = np.stack([npu4.quant_dequant(dn[e], sym=True) for e in range(E)])
    ref = moe_reference(x.numpy(), idx.numpy().astype(np.int32), wts.numpy(), Wg, Wd)
    assert_close(y, ref)
