"""Two ranks on two GPUs (skipped with fewer): the peer-memory all-reduce against the exact sums
(direct calls, calls alternating buffers, a CUDA-graph replay), the tensor-parallel decoder layer
with the row-parallel GEMVs fused with that all-reduce (one communicator per call site), and the
expert-parallel MoE layer (NCCL all-gather + reduce-scatter) against the single-GPU layer. NVLS is
off in NCCL; the peer kernels use plain peer stores."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")]


def _free_port():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _init(rank, world, port):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                         device_id=torch.device("cuda", rank))


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return dict(out)


def _allreduce_main(rank, world, port, q):
    _init(rank, world, port)
    try:
        from opennpu_b200 import libonpu as L
        from opennpu_b200.comm import PeerAllReduce
        ar = PeerAllReduce(cap_floats=1 << 14)
        errs = []
        for i, n in enumerate([5120, 37, 16384, 8, 5120 * 3]):
            vs = [torch.randn(n, generator=torch.Generator().manual_seed(100 * i + r)) for r in range(world)]
            t = vs[rank].cuda()
            ar(t)
            want = vs[0].double() + vs[1].double()
            errs.append(float((t.cpu().double() - want).abs().max()))
        # the sum as bf16 only, and as both
        v = torch.randn(4096, generator=torch.Generator().manual_seed(7 + rank)).cuda()
        vb = torch.empty(4096, device="cuda", dtype=torch.bfloat16)
        ar(v.clone(), out_bf16=vb)
        vf = torch.empty(4096, device="cuda")
        ar(v, out=vf, out_bf16=vb)
        torch.distributed.all_reduce(v)
        errs.append(float((vf - v).abs().max()))
        errs.append(float((vb.float() - v.to(torch.bfloat16).float()).abs().max()))
        # captured once, replayed with new inputs: the call counters live on the device
        x = torch.empty(5120, device="cuda")
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        x.fill_(1.0)
        with torch.cuda.stream(s):
            ar(x, stream=s)
        s.synchronize()
        with torch.cuda.graph(g, stream=s):
            ar(x, stream=s)
        for rep in range(5):
            x.fill_(float(rank + rep))
            g.replay()
            torch.cuda.synchronize()
            errs.append(float((x - float(2 * rep + 1)).abs().max()))
        del g
        torch.cuda.synchronize()
        assert L.load().onpu_check_device() == 0, L.last_error()
        torch.distributed.barrier()
        ar.close()
        torch.distributed.barrier()
        q.put((rank, max(errs)))
    finally:
        torch.distributed.destroy_process_group()


def test_peer_allreduce_two_ranks():
    res = _run(_allreduce_main)
    assert max(res.values()) <= 1e-5


def _tp_main(rank, world, port, q):
    _init(rank, world, port)
    try:
        from opennpu_b200 import tp
        from opennpu_b200.comm import PeerAllReduce
        from tests.test_tp_gpu import HIDDEN, _weights
        from oracle import oracle as O
        ars = (PeerAllReduce(cap_floats=4 * HIDDEN), PeerAllReduce(cap_floats=4 * HIDDEN))   # o, down
        w = _weights(seed=30)
        x = torch.from_numpy(O.gen_x(3, HIDDEN, seed=31)).cuda()
        lay = tp.TPDecoderLayer.from_full(w, rank, world, allreduce=ars)
        b = lay.buffers(3)
        ys = [lay(x, b).cpu().numpy() for _ in range(3)]          # both slot sets, then the first again
        torch.distributed.barrier()
        for ar in ars:
            ar.close()
        torch.distributed.barrier()
        assert all(np.array_equal(ys[0], yy) for yy in ys)
        y = ys[0]
        q.put((rank, y))
    finally:
        torch.distributed.destroy_process_group()


def test_tp_layer_peer_allreduce_two_ranks():
    from oracle import oracle as O
    from tests.test_tp_gpu import HIDDEN, _close, _oracle_layer, _weights
    res = _run(_tp_main)
    assert np.array_equal(res[0], res[1])             # both ranks hold the same sums
    x = O.gen_x(3, HIDDEN, seed=31)
    _close(res[0], _oracle_layer(_weights(seed=30), x.astype(np.float64)))


def _ep_main(rank, world, port, q):
    _init(rank, world, port)
    try:
        from opennpu_b200.moe import EPMoELayer, ExpertFFN
        from tests.test_moe_dev_gpu import _bank
        E, H, I, T = 32, 1024, 256, 6
        gq, gs = _bank(E, 2 * I, H, seed=51)
        dq, ds = _bank(E, H, I, seed=52)
        el = E // world
        sh = ExpertFFN(gq[rank * el:(rank + 1) * el], gs[rank * el:(rank + 1) * el], dq[rank * el:(rank + 1) * el],
                       ds[rank * el:(rank + 1) * el])
        g = torch.Generator(device="cuda").manual_seed(53)
        wr = (torch.randn(E, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        xs = torch.randn(world, T, H, device="cuda", generator=g).to(torch.bfloat16)
        layer = EPMoELayer(wr, sh, rank, world, E, k=8)
        y = layer(xs[rank], layer.buffers(T, H)).cpu().numpy()
        torch.distributed.barrier()
        q.put((rank, y))
    finally:
        torch.distributed.destroy_process_group()


def _ep_a2a_main(rank, world, port, q):
    _init(rank, world, port)
    try:
        from opennpu_b200.moe import EPMoELayerA2A, ExpertFFN
        from tests.test_moe_dev_gpu import _bank
        E, H, I, T = 32, 1024, 256, 6
        gq, gs = _bank(E, 2 * I, H, seed=51)
        dq, ds = _bank(E, H, I, seed=52)
        el = E // world
        sh = ExpertFFN(gq[rank * el:(rank + 1) * el], gs[rank * el:(rank + 1) * el], dq[rank * el:(rank + 1) * el],
                       ds[rank * el:(rank + 1) * el])
        g = torch.Generator(device="cuda").manual_seed(53)
        wr = (torch.randn(E, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
        xs = torch.randn(world, T, H, device="cuda", generator=g).to(torch.bfloat16)
        layer = EPMoELayerA2A(wr, sh, rank, world, E, k=8)
        y = layer(xs[rank]).cpu().numpy()
        y2 = layer(xs[rank]).cpu().numpy()
        torch.distributed.barrier()
        q.put((rank, (y, y2)))
    finally:
        torch.distributed.destroy_process_group()


def test_ep_moe_all_to_all_two_ranks_matches_single_gpu():
    """The all-to-all dispatch / combine form gives the single-GPU layer's outputs (and the same
    bits on a second call)."""
    from opennpu_b200.moe import ExpertFFN, route
    from tests.test_moe_dev_gpu import _bank
    res = _run(_ep_a2a_main)
    E, H, I, T = 32, 1024, 256, 6
    gq, gs = _bank(E, 2 * I, H, seed=51)
    dq, ds = _bank(E, H, I, seed=52)
    full = ExpertFFN(gq, gs, dq, ds)
    g = torch.Generator(device="cuda").manual_seed(53)
    wr = (torch.randn(E, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    xs = torch.randn(2, T, H, device="cuda", generator=g).to(torch.bfloat16)
    for r in range(2):
        y, y2 = res[r]
        assert np.array_equal(y, y2)
        ids, w = route(xs[r], wr, 8)
        ref = full(xs[r], ids, w).cpu().numpy()
        err = np.linalg.norm(y - ref) / np.linalg.norm(ref)
        assert err <= 1e-4, (r, err)


def test_ep_moe_layer_two_ranks_matches_single_gpu():
    from opennpu_b200.moe import ExpertFFN, route
    from tests.test_moe_dev_gpu import _bank
    res = _run(_ep_main)
    E, H, I, T = 32, 1024, 256, 6
    gq, gs = _bank(E, 2 * I, H, seed=51)
    dq, ds = _bank(E, H, I, seed=52)
    full = ExpertFFN(gq, gs, dq, ds)
    g = torch.Generator(device="cuda").manual_seed(53)
    wr = (torch.randn(E, H, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    xs = torch.randn(2, T, H, device="cuda", generator=g).to(torch.bfloat16)
    for r in range(2):
        ids, w = route(xs[r], wr, 8)
        ref = full(xs[r], ids, w).cpu().numpy()
        err = np.linalg.norm(res[r] - ref) / np.linalg.norm(ref)
        assert err <= 1e-4, (r, err)            # the shards split rows differently: last-bit differences
