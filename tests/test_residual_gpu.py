"""The two-pass (~8-bit) mode of the reference's NPULinearGroup(residual=True): W and its
quantisation residual W - quant_dequant(W), both quantised on the GPU and stored interleaved per
strip, summed in the GEMV epilogue (ONPU_EPI_PAIRSUM). Checked against the oracle (codes and
scales bit for bit, outputs within the north-star tolerance) and against the same mode through
the reference ABI (onpu_dense_mv on the stacked 2N rows, halves added on the host)."""
import numpy as np
import pytest
import torch

from opennpu_b200 import npu4
from opennpu_b200.dense import DenseMatrix, EPI_PAIRSUM
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _weights(N, K, seed):
    rng = np.random.default_rng(seed)
    return (rng.normal(0, 0.05, size=(N, K)) * rng.choice([1, 4, 0.25], size=(N, 1))).astype(np.float32)


def _gpu_order(a, N):
    """Stacked rows [W-part; R-part] (2N) -> the GPU's strip interleave (rows 0-7 of a strip from
    the first half, rows 8-15 from the second)."""
    out = np.empty_like(a)
    for rho in range(2 * N):
        strip, rr = divmod(rho, 16)
        out[rho] = a[8 * strip + rr] if rr < 8 else a[N + 8 * strip + rr - 8]
    return out


@pytest.mark.parametrize("sym", [1, 0])
def test_residual_codes_bit_exact(sym):
    N, K = 64, 512
    W = _weights(N, K, seed=3 + sym)
    m = DenseMatrix.from_float_residual(torch.from_numpy(W).cuda(), sym=bool(sym))
    q, s, mn = m.unpack()
    R = W - O.quant_dequant(W, sym)
    q1, s1, m1 = O.quantize_codes(W, sym)
    q2, s2, m2 = O.quantize_codes(R, sym)
    assert np.array_equal(q.cpu().numpy(), _gpu_order(np.concatenate([q1, q2]), N))
    assert np.array_equal(s.cpu().numpy().view(np.uint16), _gpu_order(np.concatenate([s1, s2]), N))
    if not sym:
        assert np.array_equal(mn.cpu().numpy().view(np.uint16), _gpu_order(np.concatenate([m1, m2]), N))


@pytest.mark.parametrize("sym", [1, 0])
@pytest.mark.parametrize("M", [1, 5])
def test_residual_gemv_matches_oracle_and_reference_abi(sym, M):
    N, K = 256, 1024
    W = _weights(N, K, seed=10 + sym)
    x = O.gen_x(M, K, seed=11)
    m = DenseMatrix.from_float_residual(torch.from_numpy(W).cuda(), sym=bool(sym))
    y = m.mv(torch.from_numpy(x).to(torch.bfloat16).cuda())
    assert y.shape == (M, N)
    torch.cuda.synchronize()
    y = y.cpu().numpy().astype(np.float64)
    Wq1 = O.quant_dequant(W, sym)
    Wq2 = O.quant_dequant(W - Wq1, sym)
    ref = O.matmul_xwT(x, Wq1.astype(np.float64) + Wq2.astype(np.float64)).astype(np.float64)
    err = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert err <= 1e-3, err
    assert np.abs(y - ref).max() <= 2e-2
    # ~8-bit precision: the two passes are much closer to x . W^T than one
    exact = O.matmul_xwT(x, W).astype(np.float64)
    one = O.matmul_xwT(x, Wq1).astype(np.float64)
    assert np.linalg.norm(y - exact) < 0.2 * np.linalg.norm(one - exact)
    # the reference ABI's host-summed form of the same mode
    g = npu4.NPULinearGroup(["w"], [W], sym=bool(sym), residual=True)
    yr = g.full(torch.from_numpy(x))
    err2 = np.linalg.norm(y - yr) / np.linalg.norm(yr)
    assert err2 <= 1e-3, err2


def test_residual_rejects_other_epilogues():
    from opennpu_b200 import libonpu as L
    W = _weights(64, 256, seed=20)
    m = DenseMatrix.from_float_residual(torch.from_numpy(W).cuda())
    plain = DenseMatrix.from_float(torch.from_numpy(W).cuda())
    x = torch.zeros(1, 256, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(L.OnpuError):
        plain.mv(x, epi=EPI_PAIRSUM)
    with pytest.raises(L.OnpuError):
        m.mv(x, epi=2)                                   # SwiGLU needs a gate/up matrix
