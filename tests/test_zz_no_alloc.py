"""onpu_dense_mv_dev_noalloc (static device scratch, no allocation in the call) against
onpu_dense_mv_dev on the same matrix and inputs, two calls in a row. Both entries launch the same
grid, so the split rows are added in the same order and the outputs agree bit for bit; the
regular path itself is checked against the oracle by the GEMV parity tests.

Collected last on purpose: it must pass in a fresh process (the first call sets up the static
scratch) and after every other test (the shared scratch and status word have seen other launches).
"""
import pytest
import torch

from opennpu_b200 import libonpu as L
from opennpu_b200.dense import DenseMatrix, EPI_F32, EPI_BF16, EPI_SWIGLU, EPI_SWIGLU_F32, EPI_PAIRSUM

pytestmark = pytest.mark.gpu

MAX_ROWS = 256
REL_L2, MAX_ABS = 1e-3, 2e-2          # the north-star output tolerance


def _weights(N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    qk = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
    s = (torch.randn(N, K // 32, device="cuda", generator=g).abs() * 0.02 + 1e-4).half()
    return qk, s


def _x(rows, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randn(rows, K, device="cuda", generator=g).to(torch.bfloat16)


def _call(fn, m, x, rows, epi):
    n_out = m.N // 2 if epi in (EPI_SWIGLU, EPI_SWIGLU_F32, EPI_PAIRSUM) else m.N
    bf16 = epi in (EPI_BF16, EPI_SWIGLU)
    y = torch.empty(rows, n_out, device="cuda", dtype=torch.bfloat16 if bf16 else torch.float32)
    s = torch.cuda.current_stream().cuda_stream
    rc = fn(m.h, x.data_ptr(), x.stride(0), rows, y.data_ptr(), y.stride(0), epi, s)
    L.check(rc, fn.__name__)
    return y


def _close(a, b):
    """Bit-identical (same grid and summation order), hence also within the output tolerance."""
    assert a.dtype == b.dtype and a.shape == b.shape
    assert torch.equal(a, b), (a.float() - b.float()).abs().max().item()


# (N, K, gateup, epilogue, (rows of call 1, rows of call 2))
CASES = [
    (256, 8192, False, EPI_F32, (1, 5)),            # few row groups, long K: row groups split over CTAs
    (4096, 4096, False, EPI_F32, (17, 3)),          # two MMA tiles, then one
    (1024, 2048, False, EPI_BF16, (16, 16)),
    (2048, 1024, True, EPI_SWIGLU, (1, 40)),        # fused SwiGLU, several descriptors
    (6144, 4096, True, EPI_SWIGLU_F32, (1, 8)),     # fused SwiGLU with fp32 outputs
    (4096, 12288, False, EPI_F32, (1, 2)),          # a Qwen3-8B down projection: each CTA stages its part of K
]


@pytest.mark.parametrize("N,K,gateup,epi,rows", CASES)
def test_noalloc_matches_dev_two_calls(N, K, gateup, epi, rows):
    lib = L.require_device()
    qk, s = _weights(N, K, seed=N + K)
    m = DenseMatrix.from_int4(qk, s, gateup=gateup)
    for i, r in enumerate(rows):
        x = _x(r, K, seed=100 * i + r)
        y_ref = _call(lib.onpu_dense_mv_dev, m, x, r, epi)
        y_new = _call(lib.onpu_dense_mv_dev_noalloc, m, x, r, epi)
        torch.cuda.synchronize()
        _close(y_new, y_ref)
    assert lib.onpu_check_device() == 0, L.last_error()


def test_noalloc_two_pass_pairsum():
    """The two-pass (residual) matrix and its pair-sum epilogue through both entries."""
    lib = L.require_device()
    g = torch.Generator(device="cuda").manual_seed(11)
    W = torch.randn(512, 2048, device="cuda", generator=g) * 0.05
    m = DenseMatrix.from_float_residual(W)
    for i, r in enumerate((1, 6)):
        x = _x(r, 2048, seed=50 + i)
        y_ref = _call(lib.onpu_dense_mv_dev, m, x, r, EPI_PAIRSUM)
        y_new = _call(lib.onpu_dense_mv_dev_noalloc, m, x, r, EPI_PAIRSUM)
        torch.cuda.synchronize()
        _close(y_new, y_ref)
    assert lib.onpu_check_device() == 0, L.last_error()


def test_noalloc_back_to_back_calls_share_scratch():
    """Two no-alloc calls queued back to back on one stream, then compared with the regular path."""
    lib = L.require_device()
    qk, s = _weights(512, 8192, seed=7)
    m = DenseMatrix.from_int4(qk, s)
    xa, xb = _x(3, 8192, seed=1), _x(9, 8192, seed=2)
    ya = _call(lib.onpu_dense_mv_dev_noalloc, m, xa, 3, EPI_F32)
    yb = _call(lib.onpu_dense_mv_dev_noalloc, m, xb, 9, EPI_F32)
    ra = _call(lib.onpu_dense_mv_dev, m, xa, 3, EPI_F32)
    rb = _call(lib.onpu_dense_mv_dev, m, xb, 9, EPI_F32)
    torch.cuda.synchronize()
    _close(ya, ra)
    _close(yb, rb)
    assert lib.onpu_check_device() == 0, L.last_error()


def test_noalloc_allocates_no_device_memory():
    lib = L.require_device()
    qk, s = _weights(1024, 4096, seed=3)
    m = DenseMatrix.from_int4(qk, s)
    xs = [_x(r, 4096, seed=r) for r in (1, 7, 33, 200)]
    ys = [torch.empty(x.shape[0], 1024, device="cuda") for x in xs]
    st = torch.cuda.current_stream().cuda_stream
    L.check(lib.onpu_dense_mv_dev_noalloc(m.h, xs[0].data_ptr(), 4096, 1, ys[0].data_ptr(), 1024, EPI_F32, st), "setup")
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for x, y in zip(xs, ys):     # row counts the regular path has not seen would allocate descriptors there
        L.check(lib.onpu_dense_mv_dev_noalloc(m.h, x.data_ptr(), 4096, x.shape[0], y.data_ptr(), 1024, EPI_F32, st),
                "noalloc")
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_rejects_rows_beyond_limit():
    lib = L.require_device()
    qk, s = _weights(256, 1024, seed=5)
    m = DenseMatrix.from_int4(qk, s)
    x = _x(MAX_ROWS + 1, 1024, seed=0)
    y = torch.empty(MAX_ROWS + 1, 256, device="cuda")
    rc = lib.onpu_dense_mv_dev_noalloc(m.h, x.data_ptr(), 1024, MAX_ROWS + 1, y.data_ptr(), 256, EPI_F32,
                                       torch.cuda.current_stream().cuda_stream)
    assert rc < 0
    assert "256" in L.last_error()
    # the limit itself is accepted and matches the regular path
    y_new = _call(lib.onpu_dense_mv_dev_noalloc, m, x[:MAX_ROWS], MAX_ROWS, EPI_F32)
    y_ref = _call(lib.onpu_dense_mv_dev, m, x[:MAX_ROWS], MAX_ROWS, EPI_F32)
    torch.cuda.synchronize()
    _close(y_new, y_ref)
