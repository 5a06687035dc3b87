"""GEMV chains (onpu_chain_*): a sequence of dense GEMVs run as one persistent launch, checked
link by link against the single-matrix entry point and the oracle, including links that read
another link's outputs and buffers reused across links."""
import numpy as np
import pytest
import torch

from opennpu_b200 import libonpu as L
from opennpu_b200.dense import DenseChain, DenseMatrix, EPI_BF16, EPI_F32, EPI_SWIGLU
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 1e-3, 2e-2


def _weights(N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qk = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
    s = (torch.randn(N, K // 32, device="cuda", generator=g).abs() * 0.02 + 1e-4).half()
    return qk, s


def _x(rows, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(rows, K, device="cuda", generator=g).to(torch.bfloat16)


def _close(a, b, rel=REL_L2):
    a, b = a.float(), b.float()
    err = ((a - b).norm() / b.norm().clamp_min(1e-30)).item()
    assert err <= rel, err
    assert (a - b).abs().max().item() <= MAX_ABS


@pytest.mark.parametrize("M,shapes", [
    (1, [(1024, 4096), (256, 8192), (4096, 1024), (64, 64), (3000, 992)]),
    (3, [(1024, 4096), (256, 8192), (4096, 1024), (64, 64), (3000, 992)]),
    (8, [(1024, 4096), (4096, 1024), (64, 64), (3000, 992)]),
    (9, [(1024, 2048), (4096, 1024), (64, 64), (3000, 992), (512, 2048)]),
    (16, [(512, 2048), (2048, 1024), (64, 64), (1000, 992), (128, 4096)]),
])
def test_chain_independent_links_match_oracle(M, shapes):
    chain = DenseChain()
    links = []
    for i, (N, K) in enumerate(shapes):
        v, sc = O.gen_weights(N, K, seed=i)
        m = DenseMatrix.from_int4(torch.from_numpy(O.pack_baseline(v)).cuda(),
                                  torch.from_numpy(sc.view(np.int16)).cuda())
        xf = O.gen_x(M, K, seed=10 + i)
        x, y = torch.from_numpy(xf).to(torch.bfloat16).cuda(), torch.empty(M, N, device="cuda")
        assert chain.add(m, x, y) == i
        assert chain.dep(i) == -1
        links.append((v, sc, xf, m, x, y))
    chain.run()
    torch.cuda.synchronize()
    L.check(L.load().onpu_check_device(), "device status")
    for v, sc, xf, m, x, y in links:
        ref = torch.from_numpy(O.matmul_xwT(xf, O.dequant_baseline(v, sc))).float()
        _close(y.cpu(), ref)
        _close(y, m.mv(x), rel=1e-5)


def test_chain_ffn_dependency_and_reruns():
    """gate_up (SwiGLU, bf16 out) -> down reads it: the down link waits for the whole gate_up."""
    H, I, M = 2048, 768, 4
    qg, sg = _weights(2 * I, H, seed=1)
    qd, sd = _weights(H, I, seed=2)
    gu = DenseMatrix.from_int4(qg, sg, gateup=True)
    dn = DenseMatrix.from_int4(qd, sd)
    x = _x(M, H, seed=3)
    a = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(M, H, device="cuda")
    chain = DenseChain()
    chain.add(gu, x, a, epi=EPI_SWIGLU)
    chain.add(dn, a, y)
    assert chain.dep(1) == 0
    for rep in range(3):                       # counters reset between runs
        x.copy_(_x(M, H, seed=100 + rep))
        chain.run()
        a_ref = gu.mv(x, epi=EPI_SWIGLU)
        y_ref = dn.mv(a_ref)
        torch.cuda.synchronize()
        _close(a, a_ref, rel=1e-5)
        _close(y, y_ref, rel=1e-5)
    L.check(L.load().onpu_check_device(), "device status")


def test_chain_buffer_reuse_orders_links():
    """Link 0 writes A, link 1 reads A, link 2 overwrites A, link 3 reads the new A."""
    K, N, M = 2048, 2048, 2
    mats = []
    for i in range(4):
        qk, s = _weights(N, K, seed=20 + i)
        mats.append(DenseMatrix.from_int4(qk, s))
    x0 = _x(M, K, seed=5)
    A = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    B = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    C = torch.empty(M, N, device="cuda")
    chain = DenseChain()
    chain.add(mats[0], x0, A, epi=EPI_BF16)
    chain.add(mats[1], A, B, epi=EPI_BF16)
    chain.add(mats[2], B, A, epi=EPI_BF16)
    chain.add(mats[3], A, C)
    assert [chain.dep(i) for i in range(4)] == [-1, 0, 1, 2]
    chain.run()
    torch.cuda.synchronize()
    # each link against the single-matrix path on the chain's own inputs; link 1's input (link 0's
    # A) was overwritten by link 2, so B is checked against a recomputed A: its bf16 elements may
    # round one ulp apart, so B may differ by a few bf16 ulps of its largest value
    r0 = mats[0].mv(x0, epi=EPI_BF16)
    r1 = mats[1].mv(r0, epi=EPI_BF16)
    a_ref = mats[2].mv(B, epi=EPI_BF16)
    c_ref = mats[3].mv(A)
    torch.cuda.synchronize()
    bmax = r1.float().abs().max().item()
    assert ((B.float() - r1.float()).norm() / r1.float().norm()).item() <= REL_L2
    assert (B.float() - r1.float()).abs().max().item() <= bmax * 2.0 ** -6
    assert (A.float() - a_ref.float()).abs().max().item() <= a_ref.float().abs().max().item() * 2.0 ** -8
    _close(C, c_ref, rel=1e-5)


def test_chain_decode_stack_serial():
    """Three layers of q/k/v, gate_up + SwiGLU, down with shared output buffers, every link
    ordered after its predecessor, as one decode step."""
    H, I, QKV, M = 1024, 1536, 1536, 1
    layers, chain = [], DenseChain()
    yq = torch.empty(M, QKV, device="cuda")
    a = torch.empty(M, I, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(M, H, device="cuda")
    xs, outs = [], []
    for l in range(3):
        q = DenseMatrix.from_int4(*_weights(QKV, H, seed=30 + l))
        g = DenseMatrix.from_int4(*_weights(2 * I, H, seed=40 + l), gateup=True)
        d = DenseMatrix.from_int4(*_weights(H, I, seed=50 + l))
        x = _x(M, H, seed=60 + l)
        prev = len(xs) * 3 - 1
        chain.add(q, x, yq, dep=prev)
        chain.add(g, x, a, epi=EPI_SWIGLU, dep=prev + 1)
        chain.add(d, a, y, dep=prev + 2)
        layers.append((q, g, d))
        xs.append(x)
    assert [chain.dep(i) for i in range(9)] == list(range(-1, 8))
    chain.run()
    torch.cuda.synchronize()
    q, g, d = layers[-1]
    _close(yq, q.mv(xs[-1]), rel=1e-5)
    a_ref = g.mv(xs[-1], epi=EPI_SWIGLU)
    _close(a, a_ref, rel=1e-5)
    _close(y, d.mv(a_ref), rel=1e-5)
    L.check(L.load().onpu_check_device(), "device status")


def test_chain_graph_replay_matches():
    """A chain run captured in a CUDA graph and replayed gives the same outputs as direct runs."""
    K, N, M = 4096, 2048, 1
    m = DenseMatrix.from_int4(*_weights(N, K, seed=70))
    x, y = _x(M, K, seed=71), torch.empty(M, N, device="cuda")
    chain = DenseChain()
    chain.add(m, x, y)
    chain.prepare()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        chain.run(stream=s)
    for rep in range(3):
        x.copy_(_x(M, K, seed=200 + rep))
        g.replay()
        ref = m.mv(x)
        torch.cuda.synchronize()
        _close(y, ref, rel=1e-5)
    del g


def test_chain_rejects_bad_links():
    lib = L.require_device()
    m4 = DenseMatrix.from_int4(*_weights(256, 512, seed=80))
    x = _x(17, 512, seed=81)
    y = torch.empty(17, 256, device="cuda")
    chain = DenseChain()
    rc = lib.onpu_chain_add(chain.h, m4.h, x.data_ptr(), 512, 17, y.data_ptr(), 256, EPI_F32, -1)
    assert rc < 0 and "rows" in L.last_error()
    rc = lib.onpu_chain_add(chain.h, m4.h, x.data_ptr(), 512, 1, y.data_ptr(), 256, EPI_SWIGLU, -1)
    assert rc < 0
    rc = lib.onpu_chain_add(chain.h, m4.h, x.data_ptr(), 512, 1, y.data_ptr(), 256, EPI_F32, 0)
    assert rc < 0 and "earlier" in L.last_error()
    assert chain.add(m4, x[:1], y[:1]) == 0
    # a q4s matrix (the reference's upload protocol) cannot join an int4 + fp16 chain
    N, K = 64, 512
    W = np.random.default_rng(0).standard_normal((N, K)).astype(np.float32) * 0.02
    q = DenseMatrix.from_stream(N, K, 1, O.pack(W, 8, 1))
    rc = lib.onpu_chain_add(chain.h, q.h, x.data_ptr(), 512, 1, y.data_ptr(), 256, EPI_F32, -1)
    assert rc < 0 and "format" in L.last_error()


def test_chain_rejects_activations_beyond_shared_memory():
    """Every link's activations stay resident in shared memory: 9 rows of K = 12288 do not fit,
    and the chain says so instead of running."""
    m = DenseMatrix.from_int4(*_weights(128, 12288, seed=90))
    x, y = _x(9, 12288, seed=91), torch.empty(9, 128, device="cuda")
    chain = DenseChain()
    chain.add(m, x, y)
    with pytest.raises(L.OnpuError, match="shared memory"):
        chain.prepare()


@pytest.mark.parametrize("M", [1, 8, 16])
def test_chain_runs_are_bitwise_identical(M):
    """Split row groups are reduced in contributor order, whoever arrives last: repeated runs of
    the same chain give the same bits (a race between CTAs would show up here)."""
    shapes = [(6144, 4096), (512, 8192), (4096, 12288), (96, 2048)] if M == 1 else \
        [(6144, 4096), (512, 4096), (4096, 2048), (96, 2048)]
    chain = DenseChain()
    outs = []
    for i, (N, K) in enumerate(shapes):
        m = DenseMatrix.from_int4(*_weights(N, K, seed=300 + i))
        x, y = _x(M, K, seed=310 + i), torch.empty(M, N, device="cuda")
        chain.add(m, x, y)
        outs.append((m, x, y))
    chain.run()
    torch.cuda.synchronize()
    first = [y.clone() for _, _, y in outs]
    for _ in range(4):
        chain.run()
        torch.cuda.synchronize()
        for (m, x, y), f in zip(outs, first):
            assert torch.equal(y, f)
    for (m, x, y), f in zip(outs, first):
        _close(m.mv(x), f, rel=1e-5)
    L.check(L.load().onpu_check_device(), "device status")
