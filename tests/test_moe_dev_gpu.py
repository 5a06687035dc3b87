"""Device-resident MoE layer: the router (onpu_route_dev) against the oracle's softmax / top-k /
renormalise, and the routed-expert FFN (onpu_moe_ffn_dev, int4 banks) against the oracle's
dequantise-then-matmul (opennpu/native/reference.py:77-84: fp32 activations between the
projections, never rounded), at the north-star bound rel-L2 <= 1e-3, max-abs <= 2e-2."""
import numpy as np
import pytest
import torch

from opennpu_b200 import libonpu as L
from opennpu_b200.moe import ExpertFFN, route
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 1e-3, 2e-2
W_TOL = 1e-5            # fp32 softmax vs the float64 oracle


def _router_inputs(T, E, H, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    h = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    wr = (torch.randn(E, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    return h, wr


def _check_route(ids, w, h, wr, k, norm):
    ref_ids, ref_w, ref_lg = O.route(h.float().cpu().numpy(), wr.float().cpu().numpy(), k, norm)
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    lg = ref_lg.astype(np.float64)
    prob = np.exp(lg - lg.max(-1, keepdims=True))
    prob /= prob.sum(-1, keepdims=True)
    rows = np.arange(ids.shape[0])[:, None]
    # the same probabilities in the same order: ids may differ only between near-equal experts
    assert np.abs(prob[rows, ids] - prob[rows, ref_ids]).max() <= 1e-6
    assert all(len(set(r)) == k for r in ids)
    assert np.abs(w - ref_w).max() <= W_TOL
    return ids, ref_ids


@pytest.mark.parametrize("T,E,H,k", [(1, 128, 2048, 8), (16, 128, 2048, 8), (64, 128, 2048, 8), (300, 64, 1024, 4),
                                     (5, 256, 4096, 16), (3, 40, 264, 1)])
@pytest.mark.parametrize("norm", [1, 0])
def test_route_matches_oracle(T, E, H, k, norm):
    h, wr = _router_inputs(T, E, H, seed=T + E)
    ids, w, lg = route(h, wr, k, norm_topk_prob=bool(norm), logits=True)
    torch.cuda.synchronize()
    ids, ref_ids = _check_route(ids, w, h, wr, k, norm)
    assert (ids == ref_ids).mean() > 0.99
    ref_lg = h.double() @ wr.double().T
    assert (lg.double() - ref_lg).abs().max().item() <= 1e-4


def test_route_ties_take_lower_expert_id():
    """Equal router rows give bitwise-equal logits: the lower expert id comes first (a stable
    argsort of -p, as torch.topk on the reference's CPU and the oracle)."""
    T, E, H, k = 4, 32, 512, 4
    h, wr = _router_inputs(T, E, H, seed=7)
    wr[9] = h[0] * 0.05                  # the favourite of token 0, three times over
    wr[3] = wr[9]
    wr[20] = wr[9]
    ids, w = route(h, wr, k)
    torch.cuda.synchronize()
    assert ids[0, :3].tolist() == [3, 9, 20]
    assert w[0, 0].item() == w[0, 1].item() == w[0, 2].item()
    _check_route(ids, w, h, wr, k, 1)


def test_route_full_size_properties():
    """Config-4 router at a large token count: distinct ids in range, weights descending and
    summing to one, and a sample of tokens against the oracle."""
    T, E, H, k = 8192, 128, 2048, 8
    h, wr = _router_inputs(T, E, H, seed=11)
    ids, w = route(h, wr, k)
    torch.cuda.synchronize()
    assert ids.min().item() >= 0 and ids.max().item() < E
    s, _ = ids.sort(-1)
    assert bool((s[:, 1:] != s[:, :-1]).all())
    assert bool((w[:, 1:] <= w[:, :-1]).all())
    assert (w.sum(-1) - 1).abs().max().item() <= 1e-5
    idx = torch.arange(0, T, 97, device="cuda")
    _check_route(ids[idx], w[idx], h[idx], wr, k, 1)


def test_route_rejects_bad_arguments():
    lib = L.require_device()
    h, wr = _router_inputs(2, 300, 512, seed=1)
    ids = torch.empty(2, 17, dtype=torch.int32, device="cuda")
    w = torch.empty(2, 17, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.onpu_route_dev(h.data_ptr(), 512, 2, wr.data_ptr(), 300, 512, 8, 1, ids.data_ptr(), w.data_ptr(), 0, st) < 0
    assert lib.onpu_route_dev(h.data_ptr(), 512, 2, wr.data_ptr(), 64, 512, 17, 1, ids.data_ptr(), w.data_ptr(), 0, st) < 0
    assert lib.onpu_route_dev(h.data_ptr(), 512, 2, wr.data_ptr(), 64, 500, 8, 1, ids.data_ptr(), w.data_ptr(), 0, st) < 0
    assert lib.onpu_route_dev(h.data_ptr(), 512, 2, wr.data_ptr(), 64, 512, 0, 1, ids.data_ptr(), w.data_ptr(), 0, st) < 0


# ------------------------------------------------------------------ routed-expert FFN
def _bank(E, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qk = torch.randint(0, 256, (E, N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
    s = (torch.randn(E, N, K // 32, device="cuda", generator=g).abs() * 0.02 + 1e-4).half()
    return qk, s


def _deq(qk, s):
    """uint8 [N, K/2] + fp16 [N, K/32] (CPU numpy) -> fp32 [N, K]."""
    v = O.unpack_baseline(qk, qk.shape[1] * 2)
    return O.dequant_baseline(v, s)


def _ffn_oracle(x, ids, w, gq, gs, dq, ds):
    """y[t] = sum_j w[t, j] * Wd_e . (silu(Wg_e . x_t) * (Wu_e . x_t)), float64 sums, the
    activation not rounded (reference.py:84)."""
    T, k = ids.shape
    I = gq.shape[1] // 2
    out = np.zeros((T, dq.shape[1]), np.float64)
    for e in np.unique(ids):
        rows, slots = np.nonzero(ids == e)
        Wgu = _deq(gq[e], gs[e]).astype(np.float64)
        hh = np.asarray(x[rows], np.float64) @ Wgu.T
        a = O.silu(hh[:, :I]) * hh[:, I:]
        o = a @ _deq(dq[e], ds[e]).astype(np.float64).T
        out[rows] += w[rows, slots][:, None] * o
    return out


def _assert_close(y, ref):
    y = np.asarray(y, np.float64)
    err = np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30)
    assert np.isfinite(y).all()
    assert err <= REL_L2, err
    assert np.abs(y - ref).max() <= MAX_ABS, np.abs(y - ref).max()


@pytest.fixture(scope="module")
def config4():
    """Config 4's expert shapes: E = 128, hidden 2048, expert intermediate 768."""
    E, H, I = 128, 2048, 768
    gq, gs = _bank(E, 2 * I, H, seed=1)
    dq, ds = _bank(E, H, I, seed=2)
    ffn = ExpertFFN(gq, gs, dq, ds)
    torch.cuda.synchronize()
    return ffn, gq.cpu().numpy(), gs.cpu().numpy(), dq.cpu().numpy(), ds.cpu().numpy()


@pytest.mark.parametrize("T", [1, 16, 64])
def test_moe_ffn_dev_matches_oracle(config4, T):
    ffn, gq, gs, dq, ds = config4
    g = torch.Generator(device="cuda").manual_seed(100 + T)
    x = torch.randn(T, ffn.H, device="cuda", generator=g).to(torch.bfloat16)
    wr = (torch.randn(ffn.E, ffn.H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    ids, w = route(x, wr, 8)
    y = ffn(x, ids, w)
    torch.cuda.synchronize()
    L.check(L.load().onpu_check_device(), "device status")
    ref = _ffn_oracle(x.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), gq, gs, dq, ds)
    _assert_close(y.cpu().numpy(), ref)


def test_moe_ffn_dev_skewed_routing(config4):
    """Every token routed to the same 8 experts (several full jobs per expert) and one expert
    chosen by a single token."""
    ffn, gq, gs, dq, ds = config4
    T, k = 40, 8
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(T, ffn.H, device="cuda", generator=g).to(torch.bfloat16)
    ids = torch.arange(8, dtype=torch.int32, device="cuda").repeat(T, 1) * 3
    ids[7, 7] = 127
    w = torch.rand(T, k, device="cuda", generator=g)
    w = (w / w.sum(-1, keepdim=True)).contiguous()
    y = ffn(x, ids, w)
    torch.cuda.synchronize()
    ref = _ffn_oracle(x.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), gq, gs, dq, ds)
    _assert_close(y.cpu().numpy(), ref)


def test_moe_ffn_dev_flags_bad_ids(config4):
    """An expert id outside [0, E) is found on the device: the pair is dropped, the device status
    says so, and the next calls run normally."""
    ffn = config4[0]
    lib = L.load()
    x = torch.zeros(2, ffn.H, dtype=torch.bfloat16, device="cuda")
    ids = torch.tensor([[0, 128], [1, 2]], dtype=torch.int32, device="cuda")
    w = torch.full((2, 2), 0.5, device="cuda")
    ffn(x, ids, w)
    assert lib.onpu_check_device() < 0
    assert "out of range" in L.last_error()
    ids[0, 1] = 3
    ffn(x, ids, w)
    assert lib.onpu_check_device() == 0, L.last_error()


def test_moe_layer_graph_replay(config4):
    """Router + expert FFN captured in one CUDA graph (no host round trip) and replayed on new
    tokens gives the direct calls' results."""
    ffn = config4[0]
    g = torch.Generator(device="cuda").manual_seed(21)
    T = 16
    x = torch.randn(T, ffn.H, device="cuda", generator=g).to(torch.bfloat16)
    wr = (torch.randn(ffn.E, ffn.H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    s = torch.cuda.Stream()
    ids = torch.empty(T, 8, dtype=torch.int32, device="cuda")
    w = torch.empty(T, 8, device="cuda")
    y = torch.empty(T, ffn.H, device="cuda")
    with torch.cuda.stream(s):                 # sizes the scratch outside capture
        ids, w = route(x, wr, 8, stream=s)
        ffn(x, ids, w, out=y, stream=s)
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        L.check(L.load().onpu_route_dev(x.data_ptr(), x.stride(0), T, wr.data_ptr(), ffn.E, ffn.H, 8, 1,
                                        ids.data_ptr(), w.data_ptr(), 0, s.cuda_stream), "route")
        ffn(x, ids, w, out=y, stream=s)
    for rep in range(3):
        x.copy_(torch.randn(T, ffn.H, device="cuda", generator=g).to(torch.bfloat16))
        graph.replay()
        ri, rw = route(x, wr, 8)
        ry = ffn(x, ri, rw)
        torch.cuda.synchronize()
        assert torch.equal(ids, ri) and torch.equal(w, rw)
        assert torch.equal(y, ry)
    del graph
    assert L.load().onpu_check_device() == 0, L.last_error()


def test_moe_ffn_dev_is_deterministic(config4):
    ffn = config4[0]
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(64, ffn.H, device="cuda", generator=g).to(torch.bfloat16)
    wr = (torch.randn(ffn.E, ffn.H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    ids, w = route(x, wr, 8)
    a = ffn(x, ids, w)
    b = ffn(x, ids, w)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


# ------------------------------------------------------------------ one persistent launch
@pytest.fixture
def fused_mode():
    """Set onpu_moe_set_fused for one test (0: three launches, 1: the persistent kernel)."""
    lib = L.load()
    prev = []

    def set_mode(m):
        old = lib.onpu_moe_set_fused(m)
        assert old >= 0, L.last_error()
        if not prev:
            prev.append(old)
    yield set_mode
    if prev:
        lib.onpu_moe_set_fused(prev[0])


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("T", [1, 16, 64])
def test_moe_ffn_both_forms_match_oracle(config4, fused_mode, mode, T):
    """The expert FFN as three launches (mode 0) and as one persistent launch (mode 1) against the
    unmodified oracle at config 4's shapes."""
    fused_mode(mode)
    ffn, gq, gs, dq, ds = config4
    g = torch.Generator(device="cuda").manual_seed(300 + T)
    x = torch.randn(T, ffn.H, device="cuda", generator=g).to(torch.bfloat16)
    wr = (torch.randn(ffn.E, ffn.H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    ids, w = route(x, wr, 8)
    y = ffn(x, ids, w)
    torch.cuda.synchronize()
    L.check(L.load().onpu_check_device(), "device status")
    ref = _ffn_oracle(x.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), gq, gs, dq, ds)
    _assert_close(y.cpu().numpy(), ref)


def test_moe_fused_agrees_with_three_launches(config4, fused_mode):
    """The same products in fp32 either way: the outputs agree to the last bits a split row
    group's summation order can change."""
    ffn = config4[0]
    g = torch.Generator(device="cuda").manual_seed(41)
    x = torch.randn(16, ffn.H, device="cuda", generator=g).to(torch.bfloat16)
    wr = (torch.randn(ffn.E, ffn.H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    ids, w = route(x, wr, 8)
    fused_mode(0)
    a = ffn(x, ids, w)
    fused_mode(1)
    b = ffn(x, ids, w)
    c = ffn(x, ids, w)
    torch.cuda.synchronize()
    assert torch.equal(b, c)                                  # deterministic
    assert ((a - b).norm() / a.norm()).item() <= 1e-6


def test_moe_fused_skewed_routing_and_graph_replay(config4, fused_mode):
    """The persistent kernel with several jobs per expert (every token on the same 8 experts, one
    expert chosen once) checked against the oracle, then the router + FFN captured in one CUDA
    graph and replayed: its grid-barrier counters return to zero after every launch."""
    fused_mode(1)
    ffn, gq, gs, dq, ds = config4
    T, k = 40, 8
    g = torch.Generator(device="cuda").manual_seed(6)
    x = torch.randn(T, ffn.H, device="cuda", generator=g).to(torch.bfloat16)
    ids = torch.arange(8, dtype=torch.int32, device="cuda").repeat(T, 1) * 3
    ids[7, 7] = 127
    w = torch.rand(T, k, device="cuda", generator=g)
    w = (w / w.sum(-1, keepdim=True)).contiguous()
    y = ffn(x, ids, w)
    torch.cuda.synchronize()
    ref = _ffn_oracle(x.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), gq, gs, dq, ds)
    _assert_close(y.cpu().numpy(), ref)

    T = 8
    x = torch.randn(T, ffn.H, device="cuda", generator=g).to(torch.bfloat16)
    wr = (torch.randn(ffn.E, ffn.H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    s = torch.cuda.Stream()
    yl = torch.empty(T, ffn.H, device="cuda")
    with torch.cuda.stream(s):
        _, il, wl = ffn.layer(x, wr, 8, out=yl, stream=s)
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        ffn.layer(x, wr, 8, out=yl, ids=il, w=wl, stream=s)
    for _ in range(3):
        x.copy_(torch.randn(T, ffn.H, device="cuda", generator=g).to(torch.bfloat16))
        graph.replay()
        torch.cuda.synchronize()
        ri, rw = route(x, wr, 8)
        ref = _ffn_oracle(x.float().cpu().numpy(), ri.cpu().numpy(), rw.cpu().numpy(), gq, gs, dq, ds)
        assert torch.equal(il, ri)
        _assert_close(yl.cpu().numpy(), ref)
    del graph
    assert L.load().onpu_check_device() == 0, L.last_error()


def test_moe_set_fused_rejects_bad_modes():
    lib = L.load()
    assert lib.onpu_moe_set_fused(2) == -1 and lib.onpu_moe_set_fused(-1) == -1
    assert "mode" in L.last_error()


# ------------------------------------------------------------------ expert parallelism
@pytest.mark.parametrize("world", [2, 4])
def test_moe_ffn_expert_shards_sum_to_the_full_layer(world):
    """Each rank's FFN holds E / world experts; run over every token with the global ids, the
    shards' outputs (each skipping the slots routed elsewhere) add up to the full layer."""
    E, H, I, T, k = 32, 1024, 256, 24, 8
    gq, gs = _bank(E, 2 * I, H, seed=31)
    dq, ds = _bank(E, H, I, seed=32)
    full = ExpertFFN(gq, gs, dq, ds)
    g = torch.Generator(device="cuda").manual_seed(33)
    x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    wr = (torch.randn(E, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    ids, w = route(x, wr, k)
    y_full = full(x, ids, w)
    el = E // world
    y = torch.zeros(T, H, device="cuda")
    for r in range(world):
        sh = ExpertFFN(gq[r * el:(r + 1) * el], gs[r * el:(r + 1) * el], dq[r * el:(r + 1) * el],
                       ds[r * el:(r + 1) * el])
        y += sh(x, ids, w, e0=r * el)
    torch.cuda.synchronize()
    assert L.load().onpu_check_device() == 0, L.last_error()
    # the shards' GEMVs split their rows differently from the full run's: fp32 sums differ in the
    # last bits
    err = ((y - y_full).norm() / y_full.norm()).item()
    assert err <= 1e-4, err
    ref = _ffn_oracle(x.float().cpu().numpy(), ids.cpu().numpy(), w.cpu().numpy(), gq.cpu().numpy(),
                      gs.cpu().numpy(), dq.cpu().numpy(), ds.cpu().numpy())
    _assert_close(y.cpu().numpy(), ref)


def test_moe_ffn_expert_shard_with_no_routed_tokens():
    """A shard none of whose experts was chosen contributes exact zeros."""
    E, H, I, T = 16, 512, 128, 4
    gq, gs = _bank(E, 2 * I, H, seed=41)
    dq, ds = _bank(E, H, I, seed=42)
    sh = ExpertFFN(gq[8:], gs[8:], dq[8:], ds[8:])
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    ids = torch.arange(T * 2, dtype=torch.int32, device="cuda").view(T, 2) % 8
    w = torch.full((T, 2), 0.5, device="cuda")
    y = sh(x, ids, w, e0=8)
    torch.cuda.synchronize()
    assert torch.count_nonzero(y).item() == 0
    assert L.load().onpu_check_device() == 0


@pytest.mark.parametrize("T", [1, 16, 64, 300])
def test_moe_layer_one_call_matches_route_then_ffn(config4, T):
    """onpu_moe_layer_dev (router whose last CTA builds the job lists, then the experts) gives the
    same ids, weights and outputs, bit for bit, as onpu_route_dev followed by onpu_moe_ffn_dev."""
    ffn = config4[0]
    g = torch.Generator(device="cuda").manual_seed(200 + T)
    x = torch.randn(T, ffn.H, device="cuda", generator=g).to(torch.bfloat16)
    wr = (torch.randn(ffn.E, ffn.H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    ids, w = route(x, wr, 8)
    y = ffn(x, ids, w)
    for _ in range(2):                                 # twice: the counters are left at zero
        y2, ids2, w2 = ffn.layer(x, wr, 8)
        torch.cuda.synchronize()
        assert torch.equal(ids2, ids) and torch.equal(w2, w)
        assert torch.equal(y2, y)
    assert L.load().onpu_check_device() == 0, L.last_error()

