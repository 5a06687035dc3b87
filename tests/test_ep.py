"""Expert parallelism on the CPU: the MoE layer split by experts over world-size-2 gloo ranks
(tokens and routing all-gathered, each rank's experts applied to the slots routed to them, shares
summed back) equals the single-process layer of the oracle."""
import os
import socket

import numpy as np
import torch
import torch.multiprocessing as mp

from oracle import oracle as O

E, H, I, T, K = 8, 64, 32, 5, 2


def _experts(seed=0):
    rng = np.random.default_rng(seed)
    Wg = rng.normal(0, 0.1, (E, I, H))
    Wu = rng.normal(0, 0.1, (E, I, H))
    Wd = rng.normal(0, 0.1, (E, H, I))
    return Wg, Wu, Wd


def _ffn_share(x, ids, w, Wg, Wu, Wd, e0, e1):
    """The oracle layer restricted to experts [e0, e1): slots routed elsewhere add nothing."""
    out = np.zeros((x.shape[0], Wd.shape[1]))
    for t in range(x.shape[0]):
        for j in range(ids.shape[1]):
            e = int(ids[t, j])
            if e0 <= e < e1:
                a = O.silu(Wg[e] @ x[t]) * (Wu[e] @ x[t])
                out[t] += w[t, j] * (Wd[e] @ a)
    return out


def _free_port():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        return so.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.distributed.init_process_group("gloo", rank=rank, world_size=world)
    try:
        Wg, Wu, Wd = _experts()
        rng = np.random.default_rng(100 + rank)                   # this rank's own tokens
        x = rng.normal(0, 1, (T, H))
        Wr = np.random.default_rng(7).normal(0, 0.5, (E, H))
        ids, w, _ = O.route(x, Wr, K)                             # router where the tokens live
        xs = [torch.zeros(T, H, dtype=torch.float64) for _ in range(world)]
        torch.distributed.all_gather(xs, torch.from_numpy(x))
        idl = [torch.zeros(T, K, dtype=torch.int32) for _ in range(world)]
        torch.distributed.all_gather(idl, torch.from_numpy(ids))
        wl = [torch.zeros(T, K, dtype=torch.float32) for _ in range(world)]
        torch.distributed.all_gather(wl, torch.from_numpy(w))
        x_all, ids_all, w_all = (torch.cat(v).numpy() for v in (xs, idl, wl))
        el = E // world
        share = torch.from_numpy(_ffn_share(x_all, ids_all, w_all, Wg, Wu, Wd, rank * el, (rank + 1) * el))
        torch.distributed.all_reduce(share)                       # reduce-scatter = all-reduce, then my rows
        y = share[rank * T:(rank + 1) * T].numpy()
        ref = _ffn_share(x, ids, w, Wg, Wu, Wd, 0, E)
        q.put((rank, float(np.abs(y - ref).max())))
    finally:
        torch.distributed.destroy_process_group()


def test_expert_parallel_layer_gloo_world2():
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
    assert max(res.values()) <= 1e-9


def test_plan_dispatch_sends_each_token_once_to_each_expert_rank():
    import torch
    from opennpu_b200.moe import plan_dispatch
    g = torch.Generator().manual_seed(0)
    E, k, T, world = 32, 8, 50, 4
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    order, counts = plan_dispatch(ids, E, world)
    assert int(counts.sum()) == order.numel()
    o = 0
    for d in range(world):
        toks = order[o:o + int(counts[d])].tolist()
        o += int(counts[d])
        want = [t for t in range(T) if any(int(e) // (E // world) == d for e in ids[t])]
        assert toks == want
