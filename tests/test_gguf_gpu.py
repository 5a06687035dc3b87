"""GGUF ingest on the GPU: Q4_0 and Q4_K rows -> codes, scales and mins bit-exact with the oracle
(the reference's transcode, llama/ggml-opennpu/ggml-opennpu.cpp:100-143, restated), and the dense
and expert-bank GEMVs over such weights against the oracle's dequantise-then-matmul."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "gguf.npz")
Q4_0, Q4_K = 2, 12


def _lib():
    from opennpu_b200 import libonpu as L
    return L, L.require_device()


def _rows(type_, N, K, seed):
    """N GGUF rows of K weights: golden blocks first (their edge cases), then seeded random ones."""
    rng = np.random.default_rng(seed)
    if type_ == Q4_K:
        nb, bs, gold = N * K // 256, 144, GOLD["q4k_blocks"]
    else:
        nb, bs, gold = N * K // 32, 18, GOLD["q4_0_blocks"]
    b = rng.integers(0, 256, size=(nb, bs), dtype=np.uint8)
    d = (np.abs(rng.normal(0, 0.005 if type_ == Q4_K else 0.02, nb)) + 1e-4).astype(np.float16)
    b[:, 0:2] = d.view(np.uint8).reshape(nb, 2)
    if type_ == Q4_K:
        b[:, 2:4] = np.abs(rng.normal(0, 0.005, nb)).astype(np.float16).view(np.uint8).reshape(nb, 2)
    n = min(nb, gold.shape[0])
    b[:n] = gold[:n]
    return b.reshape(N, -1)


def _oracle_codes(type_, rows, N, K):
    if type_ == Q4_K:
        q, s, m = O.q4k_transcode(rows.reshape(-1, 144))
        return q.reshape(N, K), s.reshape(N, K // 32), m.reshape(N, K // 32)
    q, d = O.q4_0_codes(rows.reshape(-1, 18))
    return q.reshape(N, K), d.reshape(N, K // 32), None


def _oracle_weights(type_, q, s, m):
    N, K = q.shape
    qf = q.reshape(N, K // 32, 32).astype(np.float32)
    if type_ == Q4_K:
        w = qf * O.bf16_bits_to_f32(s)[..., None] + O.bf16_bits_to_f32(m)[..., None]
    else:
        w = (qf - 8) * s.view(np.float16).astype(np.float32)[..., None]
    return w.reshape(N, K)


@pytest.mark.parametrize("type_,N,K", [(Q4_K, 96, 256), (Q4_K, 130, 2048), (Q4_0, 96, 32), (Q4_0, 257, 5120)])
def test_gguf_codes_bit_exact(type_, N, K):
    L, lib = _lib()
    rows = _rows(type_, N, K, seed=N + K)
    src = torch.from_numpy(rows).cuda()
    q = torch.empty(N, K, dtype=torch.uint8, device="cuda")
    s = torch.empty(N, K // 32, dtype=torch.int16, device="cuda")
    m = torch.empty(N, K // 32, dtype=torch.int16, device="cuda")
    L.check(lib.onpu_gguf_codes_dev(type_, src.data_ptr(), N, K, q.data_ptr(), s.data_ptr(),
                                    m.data_ptr() if type_ == Q4_K else None, torch.cuda.current_stream().cuda_stream),
            "onpu_gguf_codes_dev")
    torch.cuda.synchronize()
    oq, os_, om = _oracle_codes(type_, rows, N, K)
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), os_)
    if type_ == Q4_K:
        assert np.array_equal(m.cpu().numpy().view(np.uint16), om)


@pytest.mark.parametrize("type_,N,K,M,gateup", [(Q4_K, 1024, 4096, 1, False), (Q4_K, 256, 2048, 5, True),
                                                (Q4_0, 4096, 4096, 1, False), (Q4_0, 512, 1536, 9, False)])
@pytest.mark.parametrize("on_device", [0, 1])
def test_dense_from_gguf_matches_oracle(type_, N, K, M, gateup, on_device):
    L, lib = _lib()
    from opennpu_b200.dense import DenseMatrix, EPI_F32, EPI_SWIGLU_F32
    rows = _rows(type_, N, K, seed=7 * N + K)
    data = torch.from_numpy(rows).cuda() if on_device else torch.from_numpy(rows)
    h = lib.onpu_dense_new_gguf(N, K, type_, data.data_ptr(), on_device, int(gateup),
                                torch.cuda.current_stream().cuda_stream)
    L.check(h, "onpu_dense_new_gguf")
    m = DenseMatrix(h, N, K, 0 if type_ == Q4_K else 2, gateup=gateup)
    W = _oracle_weights(type_, *_oracle_codes(type_, rows, N, K))
    x = O.gen_x(M, K, seed=M)
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    if gateup:
        y = m.mv(xt, epi=EPI_SWIGLU_F32).cpu().numpy().astype(np.float64)
        hh = O.matmul_xwT(x, W).astype(np.float64)
        ref = O.silu(hh[:, :N // 2]) * hh[:, N // 2:]
    else:
        y = m.mv(xt, epi=EPI_F32).cpu().numpy().astype(np.float64)
        ref = O.matmul_xwT(x, W).astype(np.float64)
    err = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert err <= 1e-5 and np.abs(y - ref).max() <= 2e-2, err
    assert lib.onpu_check_device() == 0


@pytest.mark.parametrize("type_", [Q4_K, Q4_0])
def test_bank_from_gguf_matches_oracle(type_):
    """An expert bank from a ggml [K, N, E] tensor of GGUF rows, run through the reference ABI's
    grouped expert GEMV (onpu_bank_run)."""
    L, lib = _lib()
    E, N, K, T, k = 6, 256, 512, 3, 2
    rows = _rows(type_, E * N, K, seed=11 + type_)
    h = lib.onpu_bank_new_gguf(N, K, E, type_, torch.from_numpy(rows).data_ptr(), 0, 0, None)
    L.check(h, "onpu_bank_new_gguf")
    W = _oracle_weights(type_, *_oracle_codes(type_, rows, E * N, K)).reshape(E, N, K)
    rng = np.random.default_rng(3)
    x = O.round_bf16(rng.normal(0, 1, size=(T, K)).astype(np.float32))
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    y = np.empty((T, k, N), np.float32)
    lib.onpu_bank_run(h, L.fp(x), 0, T, L.i32p(ids), k, L.fp(y))
    assert L.last_error() is None
    for t in range(T):
        for j in range(k):
            ref = O.matmul_xwT(x[t][None], W[ids[t, j]])[0]
            assert np.linalg.norm(y[t, j] - ref) <= 1e-5 * np.linalg.norm(ref)
    lib.onpu_bank_free(h)


def test_gguf_rejects_bad_layouts():
    L, lib = _lib()
    buf = torch.zeros(1 << 16, dtype=torch.uint8)
    assert lib.onpu_dense_new_gguf(64, 128, Q4_K, buf.data_ptr(), 0, 0, None) is None     # K % 256
    assert "not a supported GGUF layout" in L.last_error()
    assert lib.onpu_dense_new_gguf(64, 48, Q4_0, buf.data_ptr(), 0, 0, None) is None      # K % 32
    assert lib.onpu_dense_new_gguf(64, 256, 8, buf.data_ptr(), 0, 0, None) is None        # Q8_0: not taken
