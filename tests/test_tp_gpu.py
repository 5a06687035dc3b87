"""Tensor-parallel decoder-layer projections on the GPU: the ranks' shards (column-parallel q/k/v
and gate/up, row-parallel o and down) run through the int4 GEMV, their row-parallel partials are
summed, and the layer output matches the oracle's dequantise-then-matmul of the full matrices
(opennpu/native/reference.py:55-57, :84: fp32 activations between the projections, never
rounded). One GPU emulates the ranks (the partial sums are added by the test, in rank order); with
two or more GPUs, two NCCL ranks run the same layer."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from opennpu_b200 import tp
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HIDDEN, INTER, QH, KVH = 1024, 2048, 8, 2
REL_L2, MAX_ABS = 1e-3, 2e-2


def _weights(seed, hidden=HIDDEN, inter=INTER, qh=QH, kvh=KVH):
    w = {}
    for i, (name, N, K) in enumerate(tp.dense_layer_shapes(hidden, inter, qh, kvh)):
        v, s = O.gen_weights(N, K, seed=seed + i)
        w[name] = (torch.from_numpy(O.pack_baseline(v)), torch.from_numpy(s.view(np.int16)))
    return w


def _deq(qk, s):
    qk, s = qk.numpy(), s.numpy().view(np.float16)
    return O.dequant_baseline(O.unpack_baseline(qk, qk.shape[1] * 2), s)


def _mm(x, wq):
    """x @ W.T in float64 for a (codes, scales) matrix, dequantised a block of rows at a time."""
    qk, s = wq
    rows = max(1, (1 << 22) // (qk.shape[1] * 2))
    out = []
    for r0 in range(0, qk.shape[0], rows):
        out.append(x @ _deq(qk[r0:r0 + rows], s[r0:r0 + rows]).astype(np.float64).T)
    return np.concatenate(out, axis=1)


def _oracle_layer(w, x):
    """The layer's data flow on the full matrices (o reads the q projection's output as the
    attention stand-in), float64 sums, no rounding between the projections."""
    q = _mm(x, w["q"])
    h = _mm(q, w["o"])
    g, u = _mm(h, w["gate"]), _mm(h, w["up"])
    return _mm(O.silu(g) * u, w["down"])


def _close(y, ref):
    """rel-L2 <= 1e-3, and max-abs <= 2e-2 at the scale of one projection's output on N(0, 1)
    inputs (rms ~10): this synthetic chain has no normalisation between the projections, so its
    values grow ~10x per projection (to ~1e6 at the Qwen2.5-32B sizes) and the absolute bound is
    scaled by the output's rms / 10."""
    y = np.asarray(y, np.float64)
    assert np.isfinite(y).all()
    err = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    rms = float(np.sqrt(np.mean(ref ** 2)))
    mx = float(np.abs(y - ref).max())
    assert err <= REL_L2, (err, mx, rms)
    assert mx <= MAX_ABS * max(1.0, rms / 10.0), (err, mx, rms)


def _run_emulated(w, x, world, hidden):
    M = x.shape[0]
    layers = [tp.TPDecoderLayer.from_full(w, r, world) for r in range(world)]
    bufs = [lay.buffers(M) for lay in layers]
    h = torch.zeros(M, hidden, device="cuda")
    for lay, b in zip(layers, bufs):                     # o partials, summed in rank order
        lay.qkv(x, b["qkv"], epi=tp.EPI_F32)
        h += lay.o(b["qkv"][:, :lay.nq], b["h"])
    y = torch.zeros(M, hidden, device="cuda")
    for lay, b in zip(layers, bufs):
        lay.gu(h, b["a"], epi=tp.EPI_SWIGLU_F32)
        y += lay.dn(b["a"], b["y"])
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("M", [1, 3, 8])
def test_tp_layer_emulated_ranks_match_oracle(world, M):
    w = _weights(seed=10)
    x = torch.from_numpy(O.gen_x(M, HIDDEN, seed=11 + M)).cuda()        # fp32 activations (bf16 values)
    y = _run_emulated(w, x, world, HIDDEN)
    _close(y, _oracle_layer(w, x.cpu().numpy().astype(np.float64)))


def test_tp_layer_whole_call_matches_oracle():
    """TPDecoderLayer.__call__ itself at one rank (no communicator): fp32 input, fp32 output."""
    w = _weights(seed=30)
    x = torch.from_numpy(O.gen_x(2, HIDDEN, seed=31)).cuda()
    lay = tp.TPDecoderLayer.from_full(w, 0, 1)
    y = lay(x, lay.buffers(2))
    torch.cuda.synchronize()
    _close(y.cpu().numpy(), _oracle_layer(w, x.cpu().numpy().astype(np.float64)))


@pytest.mark.parametrize("world", [1, 8])
def test_tp_layer_qwen25_32b_shapes(world):
    """BASELINE configs[4] at full size: hidden 5120, intermediate 27648, 40 / 8 heads x 128, one
    decode token, the ranks' shards of TP = 1 and TP = 8 (K blocks of 640 and 3456)."""
    w = _weights(seed=40, hidden=5120, inter=27648, qh=40, kvh=8)
    x = torch.from_numpy(O.gen_x(1, 5120, seed=41)).cuda()
    y = _run_emulated(w, x, world, 5120)
    _close(y, _oracle_layer(w, x.cpu().numpy().astype(np.float64)))


def _free_port():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import datetime
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                         device_id=torch.device("cuda", rank))
    try:
        w = _weights(seed=20)
        M = 2
        x = torch.from_numpy(O.gen_x(M, HIDDEN, seed=21)).cuda()
        lay = tp.TPDecoderLayer.from_full(w, rank, world, group=torch.distributed.group.WORLD)
        y = lay(x, lay.buffers(M))
        torch.cuda.synchronize()
        if rank == 0:
            q.put(y.cpu().numpy())
        torch.distributed.barrier()
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_layer_two_ranks_nccl():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    y = q.get(timeout=240)
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    w = _weights(seed=20)
    x = O.gen_x(2, HIDDEN, seed=21)
    _close(y, _oracle_layer(w, x.astype(np.float64)))


@pytest.mark.parametrize("world", [1, 2, 4])
def test_tp_prefill_mlp_emulated_ranks(world):
    """Prefill under tensor parallelism on one GPU: each rank's gate/up rows and down K block on
    the tensor cores, the row-parallel partials summed in rank order, against the oracle's
    dequantise-then-matmul with the same roundings as the GPU path (fp16 weights and activations
    into the GEMMs, the SwiGLU activation rounded to bf16 between them)."""
    H, I, M = 1024, 2048, 96
    w = {}
    for i, (name, N, K) in enumerate([("gate", I, H), ("up", I, H), ("down", H, I)]):
        v, s = O.gen_weights(N, K, seed=60 + i)
        w[name] = (torch.from_numpy(O.pack_baseline(v)), torch.from_numpy(s.view(np.int16)))
    x = torch.from_numpy(O.gen_x(M, H, seed=63)).to(torch.bfloat16).cuda()
    y = torch.zeros(M, H, device="cuda")
    for r in range(world):
        mlp = tp.TPMLP.from_full(w["gate"], w["up"], w["down"], r, world)
        a = torch.empty(M, I // world, device="cuda", dtype=torch.bfloat16)
        yr = torch.empty(M, H, device="cuda")
        y += mlp(x, a, yr)
    torch.cuda.synchronize()
    f16 = lambda W: W.astype(np.float16).astype(np.float64)
    xd = x.float().cpu().numpy().astype(np.float64)
    g, u = xd @ f16(_deq(*w["gate"])).T, xd @ f16(_deq(*w["up"])).T
    a = O.round_bf16((O.silu(g) * u).astype(np.float32)).astype(np.float64)
    ref = a @ f16(_deq(*w["down"])).T
    yy = y.cpu().numpy().astype(np.float64)
    err = np.linalg.norm(yy - ref) / np.linalg.norm(ref)
    assert err <= 1e-3, err
