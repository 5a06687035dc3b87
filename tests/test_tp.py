"""Tensor-parallel sharding of the int4 projections, on the CPU: shards computed with the oracle
(dequantise-then-matmul) reproduce the full matrix (column blocks concatenate, row-block partials
sum), and a world-size-2 gloo process group all-reduces the row-parallel partials to the full
result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from opennpu_b200 import tp
from oracle import oracle as O


def _mat(N, K, seed):
    v, s = O.gen_weights(N, K, seed=seed)
    return torch.from_numpy(O.pack_baseline(v)), torch.from_numpy(s.view(np.int16)), v, s


def _deq(qk, s):
    qk, s = qk.numpy(), s.numpy().view(np.float16)
    return O.dequant_baseline(O.unpack_baseline(qk, qk.shape[1] * 2), s)


def test_split_range_rejects_uneven_splits():
    assert tp.split_range(5120, 3, 8, 32) == (1920, 2560)
    assert tp.split_range(27648, 7, 8, 32) == (24192, 27648)
    with pytest.raises(ValueError):
        tp.split_range(5120, 0, 3, 32)
    with pytest.raises(ValueError):
        tp.split_range(96, 0, 4, 32)            # 24-column blocks would cut a scale group


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_column_and_row_shards_reproduce_the_full_product(world):
    N, K = 256, 1024
    qk, s, v, sc = _mat(N, K, seed=world)
    x = O.gen_x(3, K, seed=1)
    full = O.matmul_xwT(x, O.dequant_baseline(v, sc))
    cols = [O.matmul_xwT(x, _deq(*tp.column_shard(qk, s, r, world))) for r in range(world)]
    np.testing.assert_array_equal(np.concatenate(cols, axis=1), full)
    parts = []
    for r in range(world):
        k0, k1 = tp.split_range(K, r, world, 32)
        parts.append(O.matmul_xwT(x[:, k0:k1], _deq(*tp.row_shard(qk, s, r, world)), acc=np.float64))
    np.testing.assert_allclose(np.sum(parts, axis=0), full, rtol=1e-5, atol=1e-4)


def test_fused_rows_shard_keeps_each_parts_block():
    q = _mat(64, 256, 1)[:2]
    k = _mat(32, 256, 2)[:2]
    v = _mat(32, 256, 3)[:2]
    for r in range(2):
        qk, s = tp.fused_rows_shard([q, k, v], r, 2)
        assert qk.shape == (64, 128) and s.shape == (64, 8)
        assert torch.equal(qk[:32], q[0][32 * r:32 * r + 32])
        assert torch.equal(qk[32:48], k[0][16 * r:16 * r + 16])
        assert torch.equal(s[48:], v[1][16 * r:16 * r + 16])


def test_layer_shapes_of_the_tp_configs():
    sh = dict((n, (N, K)) for n, N, K in tp.dense_layer_shapes(5120, 27648, 40, 8))
    assert sh["q"] == (5120, 5120) and sh["k"] == (1024, 5120) and sh["o"] == (5120, 5120)
    assert sh["down"] == (5120, 27648)
    assert sum(N * K for N, K in sh.values()) == 487_587_840
    for world in (2, 4, 8):
        for n in ("o", "down"):
            tp.split_range(sh[n][1], 0, world, 32)       # K blocks stay on scale-group boundaries


def _free_port():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        N, K = 128, 512
        qk, s, v, sc = _mat(N, K, seed=7)
        x = O.gen_x(2, K, seed=8)
        k0, k1 = tp.split_range(K, rank, world, 32)
        part = torch.from_numpy(O.matmul_xwT(x[:, k0:k1], _deq(*tp.row_shard(qk, s, rank, world))))
        torch.distributed.all_reduce(part)
        full = O.matmul_xwT(x, O.dequant_baseline(v, sc))
        q.put((rank, float(np.abs(part.numpy() - full).max())))
    finally:
        torch.distributed.destroy_process_group()


def test_row_parallel_all_reduce_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert max(res.values()) <= 1e-4
