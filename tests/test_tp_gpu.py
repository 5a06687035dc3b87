"""Tensor-parallel decoder-layer projections on the GPU: the ranks' shards (column-parallel q/k/v
and gate/up, row-parallel o and down) run through the int4 GEMV, their row-parallel partials are
summed, and the layer output matches the oracle's dequantise-then-matmul of the full matrices
(bf16 intermediates at the same points). One GPU emulates the ranks (the partial sums are added
by the test, in rank order); with two or more GPUs, two NCCL ranks run the same layer."""
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


def _weights(seed):
    w = {}
    for i, (name, N, K) in enumerate(tp.dense_layer_shapes(HIDDEN, INTER, QH, KVH)):
        v, s = O.gen_weights(N, K, seed=seed + i)
        w[name] = (torch.from_numpy(O.pack_baseline(v)), torch.from_numpy(s.view(np.int16)))
    return w


def _deq(qk, s):
    qk, s = qk.numpy(), s.numpy().view(np.float16)
    return O.dequant_baseline(O.unpack_baseline(qk, qk.shape[1] * 2), s).astype(np.float64)


def _oracle_layer(w, x):
    """The layer's data flow on the full matrices, float64 sums, bf16 where the GPU path rounds."""
    q = O.round_bf16((x @ _deq(*w["q"]).T).astype(np.float32)).astype(np.float64)
    h = q @ _deq(*w["o"]).T
    x2 = O.round_bf16(h.astype(np.float32)).astype(np.float64)
    g, u = x2 @ _deq(*w["gate"]).T, x2 @ _deq(*w["up"]).T
    a = O.round_bf16((O.silu(g) * u).astype(np.float32)).astype(np.float64)
    return a @ _deq(*w["down"]).T


def _close(y, ref):
    y = np.asarray(y, np.float64)
    err = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    assert err <= 1e-3, err
    # bf16 intermediates may round one ulp apart between the paths
    assert np.abs(y - ref).max() <= 2e-2 + np.abs(ref).max() * 2.0 ** -7


@pytest.mark.parametrize("world", [1, 2, 4])
def test_tp_layer_emulated_ranks_match_oracle(world):
    w = _weights(seed=10)
    M = 3
    x = torch.from_numpy(O.gen_x(M, HIDDEN, seed=11)).to(torch.bfloat16).cuda()
    layers = [tp.TPDecoderLayer.from_full(w, r, world) for r in range(world)]
    bufs = [lay.buffers(M) for lay in layers]
    h = torch.zeros(M, HIDDEN, device="cuda")
    for lay, b in zip(layers, bufs):                     # o partials, summed in rank order
        lay.qkv(x, b["qkv"], epi=tp.EPI_BF16)
        h += lay.o(b["qkv"][:, :lay.nq], b["h"])
    x2 = h.to(torch.bfloat16)
    y = torch.zeros(M, HIDDEN, device="cuda")
    for lay, b in zip(layers, bufs):
        lay.gu(x2, b["a"], epi=tp.EPI_SWIGLU)
        y += lay.dn(b["a"], b["y"])
    torch.cuda.synchronize()
    _close(y.cpu().numpy(), _oracle_layer(w, x.float().cpu().numpy().astype(np.float64)))


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
        x = torch.from_numpy(O.gen_x(M, HIDDEN, seed=21)).to(torch.bfloat16).cuda()
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
    _close(y, _oracle_layer(w, O.round_bf16(x).astype(np.float64)))
