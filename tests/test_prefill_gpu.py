"""Prefill dequant-GEMM (onpu_dense_mm_dev: tcgen05 tensor cores, fp16 operands, fp32 accumulators
in tensor memory) against the oracle's dequantise-then-matmul, at the north-star tolerance."""
import numpy as np
import pytest
import torch

from opennpu_b200 import libonpu as L
from opennpu_b200.dense import DenseMatrix, EPI_BF16, EPI_F32, EPI_SWIGLU
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2, MAX_ABS = 1e-3, 2e-2


def _assert_close(y, ref, rel=REL_L2, atol=MAX_ABS):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    assert np.isfinite(y).all()
    err = np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30)
    assert err <= rel, err
    assert np.abs(y - ref).max() <= atol, np.abs(y - ref).max()


def _int4(N, K, seed):
    v, s = O.gen_weights(N, K, seed=seed)
    m = DenseMatrix.from_int4(torch.from_numpy(O.pack_baseline(v)).cuda(), torch.from_numpy(s.view(np.int16)).cuda())
    return v, s, m


# (N, K, M): exact tiles, ragged tokens, ragged rows (not a multiple of the 256-row tile nor of
# 64), K with a half chunk at the end, one token, and a config-3-like slice
SHAPES = [(256, 256, 128), (512, 1024, 200), (300, 544, 77), (130, 160, 1), (96, 992, 129),
          (1024, 4096, 512), (4096, 1024, 130)]


@pytest.mark.parametrize("N,K,M", SHAPES)
def test_prefill_int4_matches_oracle(N, K, M):
    v, s, m = _int4(N, K, seed=N + K)
    x = O.gen_x(M, K, seed=M)
    y = m.mm(torch.from_numpy(x).to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    L.check(L.load().onpu_check_device(), "device status")
    _assert_close(y.cpu().numpy(), O.matmul_xwT(x, O.dequant_baseline(v, s)))


@pytest.mark.parametrize("sym", [0, 1])
def test_prefill_reference_formats(sym):
    """q4nx (scale + min) and q4s uploaded through the reference protocol."""
    N, K, M = 320, 512, 150
    W = (np.random.default_rng(3).standard_normal((N, K)) * 0.02).astype(np.float32)
    packed = O.pack(W, 8, sym)
    m = DenseMatrix.from_stream(N, K, sym, packed)
    q, sc, mn = O.unpack_codes(packed, N, K, 8, sym)
    Wd = O.dequant(q, sc, mn, O.FMT_Q4S if sym else O.FMT_Q4NX)[:, :K]
    x = O.gen_x(M, K, seed=4)
    y = m.mm(torch.from_numpy(x).to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    _assert_close(y.cpu().numpy(), O.matmul_xwT(x, Wd))


def test_prefill_epilogues_match_gemv():
    """bf16 and fused SwiGLU outputs of the GEMM agree with the GEMV path's (fp32 sums of exact
    products) within one bf16 rounding."""
    H, I, M = 1024, 768, 40
    v, s = O.gen_weights(2 * I, H, seed=9)
    gu = DenseMatrix.from_int4(torch.from_numpy(O.pack_baseline(v)).cuda(),
                               torch.from_numpy(s.view(np.int16)).cuda(), gateup=True)
    x = torch.from_numpy(O.gen_x(M, H, seed=10)).to(torch.bfloat16).cuda()
    for epi in (EPI_SWIGLU, EPI_BF16, EPI_F32):
        a = gu.mm(x, epi=epi).float()
        b = gu.mv(x[:16], epi=epi).float()
        torch.cuda.synchronize()
        ref = b.cpu().numpy()
        tol = MAX_ABS + float(np.abs(ref).max()) * 2.0 ** -8
        _assert_close(a[:16].cpu().numpy(), ref, rel=2e-3, atol=tol)


def test_prefill_token_beyond_fp16_range():
    """A token with |x| above the fp16 range is copied scaled by a power of two and unscaled in the
    epilogue: its outputs stay finite and within tolerance."""
    N, K, M = 256, 512, 3
    v, s, m = _int4(N, K, seed=11)
    x = O.gen_x(M, K, seed=12)
    x[1] *= 2.0 ** 18                    # bf16-exact scaling, max |x| ~ 1e6
    y = m.mm(torch.from_numpy(x).to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    ref = O.matmul_xwT(x, O.dequant_baseline(v, s))
    for t in range(M):
        _assert_close(y[t].cpu().numpy(), ref[t], atol=MAX_ABS * max(1.0, float(np.abs(ref[t]).max())))


def test_prefill_is_deterministic_and_reuses_scratch():
    v, s, m = _int4(1024, 2048, seed=13)
    xs = [torch.from_numpy(O.gen_x(M, 2048, seed=M)).to(torch.bfloat16).cuda() for M in (300, 64, 300)]
    ys = [m.mm(x) for x in xs]
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[2])
    L.check(L.load().onpu_check_device(), "device status")


def test_prefill_rejects_bad_arguments():
    lib = L.require_device()
    _, _, m = _int4(256, 512, seed=14)
    x = torch.zeros(4, 512, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(4, 256, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.onpu_dense_mm_dev(m.h, x.data_ptr(), 500, 4, y.data_ptr(), 256, EPI_F32, st) < 0
    assert lib.onpu_dense_mm_dev(m.h, x.data_ptr(), 512, 4, y.data_ptr(), 128, EPI_F32, st) < 0
    assert lib.onpu_dense_mm_dev(m.h, x.data_ptr(), 512, 4, y.data_ptr(), 256, EPI_SWIGLU, st) < 0


@pytest.fixture(scope="module")
def qwen3_14b_mlp():
    """BASELINE configs[2] at full size: gate/up 17408 x 5120 (one of the pair) and down
    5120 x 17408, int4 group-32 weights."""
    vg, sg, mg = _int4(17408, 5120, seed=141)
    vd, sd, md = _int4(5120, 17408, seed=142)
    return (vg, sg, mg), (vd, sd, md)


@pytest.mark.parametrize("M", [512, 2048])
@pytest.mark.parametrize("which", ["gate", "down"])
def test_prefill_qwen3_14b_full_size(qwen3_14b_mlp, M, which):
    """The tensor-core GEMM at config 3's shapes against the oracle's fp32 dequantise-then-matmul
    (the weights rounded to fp16 once on the GPU: ~2^-12 of each weight, within the bound). The
    oracle's product runs in fp32 BLAS here (float64 would take minutes at this size)."""
    v, s, m = qwen3_14b_mlp[0] if which == "gate" else qwen3_14b_mlp[1]
    K = v.shape[1]
    x = O.gen_x(M, K, seed=M + K)
    y = m.mm(torch.from_numpy(x).to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    L.check(L.load().onpu_check_device(), "device status")
    ref = O.matmul_xwT(x, O.dequant_baseline(v, s), acc=np.float32)
    _assert_close(y.cpu().numpy(), ref)
