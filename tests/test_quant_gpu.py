"""The load-time search quantisers on the GPU (onpu_quantize_dev, DenseMatrix.from_float) against
the oracle's C restatement of the reference's quantisers (itself bit-exact with the reference's
own libonpu host code): codes, bf16 scales and mins bit for bit, including constant, all-zero,
negative-peak, huge and tiny groups."""
import numpy as np
import pytest
import torch

from opennpu_b200 import libonpu as L
from opennpu_b200.dense import DenseMatrix
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _weights(N, K, seed):
    rng = np.random.default_rng(seed)
    W = (rng.normal(0, 0.05, size=(N, K)) * rng.choice([1, 1, 10, 1e-3], size=(N, 1))).astype(np.float32)
    W[0, :32] = 0.0                        # all zero
    W[1, 32:64] = -0.25                    # constant
    W[2, :32] = rng.normal(0, 1e-30, 32)   # tiny (denormal-range products)
    W[3, :32] *= 1e6                       # huge
    W[4, 5] = -3.0                         # a negative peak
    W[5, :32] = np.linspace(-1, 1, 32)     # exact grid ties
    return W


def _quant_gpu(W, sym):
    N, K = W.shape
    Wd = torch.from_numpy(W).cuda()
    q = torch.empty(N, K, dtype=torch.uint8, device="cuda")
    s = torch.empty(N, K // 32, dtype=torch.int16, device="cuda")
    m = torch.zeros(N, K // 32, dtype=torch.int16, device="cuda")
    rc = L.load().onpu_quantize_dev(Wd.data_ptr(), K, N, K, int(sym), q.data_ptr(), s.data_ptr(), m.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    L.check(rc, "onpu_quantize_dev")
    torch.cuda.synchronize()
    return q.cpu().numpy(), s.cpu().numpy().view(np.uint16), m.cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("sym", [1, 0])
@pytest.mark.parametrize("shape", [(70, 320), (8, 4096), (257, 96)])
def test_gpu_quantiser_bit_exact(sym, shape):
    W = _weights(*shape, seed=sum(shape) + sym)
    q, s, m = _quant_gpu(W, sym)
    rq, rs, rm = O.quantize_codes(W, sym)
    assert np.array_equal(q, rq)
    assert np.array_equal(s, rs)
    if not sym:
        assert np.array_equal(m, rm)


@pytest.mark.parametrize("sym", [1, 0])
def test_dense_from_float_matches_host_packer(sym):
    N, K = 192, 1024
    W = _weights(N, K, seed=40 + sym)
    m = DenseMatrix.from_float(torch.from_numpy(W).cuda(), sym=bool(sym))
    q, s, mn = m.unpack()
    rq, rs, rm = O.quantize_codes(W, sym)
    assert np.array_equal(q.cpu().numpy(), rq)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), rs)
    if not sym:
        assert np.array_equal(mn.cpu().numpy().view(np.uint16), rm)
    x = O.gen_x(3, K, seed=41)
    y = m.mv(torch.from_numpy(x).to(torch.bfloat16).cuda())
    torch.cuda.synchronize()
    Wq = O.quant_dequant(W, sym)
    ref = O.matmul_xwT(x, Wq)
    err = np.linalg.norm(y.cpu().numpy() - ref) / np.linalg.norm(ref)
    assert err <= 1e-3, err


def test_quantiser_rejects_bad_shapes():
    lib = L.require_device()
    W = torch.zeros(4, 48, device="cuda")
    q = torch.empty(4, 48, dtype=torch.uint8, device="cuda")
    s = torch.empty(4, 2, dtype=torch.int16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.onpu_quantize_dev(W.data_ptr(), 48, 4, 48, 1, q.data_ptr(), s.data_ptr(), 0, st) < 0
    assert lib.onpu_quantize_dev(W.data_ptr(), 30, 4, 32, 1, q.data_ptr(), s.data_ptr(), 0, st) < 0
