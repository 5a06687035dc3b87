"""A bounded wait that runs out, on one GPU and without a fault: this process is rank 0 of a
two-rank communicator whose rank 1 (a child process on the same GPU) allocates and exports its
buffer but never stores and never launches a kernel. Rank 0's fused all-reduce GEMV sends its
words and then waits for rank 1's; with the wait shortened to 0.2 s the CTAs give up, set device
status 16 and return. The library then reports an all-reduce timeout, the status is cleared, and
the next GEMV on the same context matches the oracle."""
import multiprocessing as mp

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _silent_rank(q_out, q_in):
    """Rank 1: a buffer exported to rank 0, then nothing until told to exit."""
    import ctypes as C
    from opennpu_b200 import libonpu as L
    lib = L.require_device()
    h = lib.onpu_comm_new(1, 2, 4096)
    hb = (C.c_ubyte * 64)()
    L.check(lib.onpu_comm_ipc_handle(h, hb), "onpu_comm_ipc_handle")
    q_out.put(bytes(hb))
    q_in.get(timeout=300)
    lib.onpu_comm_free(h)


def test_peer_wait_runs_out_and_the_gpu_stays_usable():
    import ctypes as C
    from opennpu_b200 import libonpu as L
    from opennpu_b200.dense import DenseMatrix
    lib = L.require_device()
    ctx = mp.get_context("spawn")
    q_out, q_in = ctx.Queue(), ctx.Queue()
    child = ctx.Process(target=_silent_rank, args=(q_out, q_in))
    child.start()
    try:
        peer_handle = q_out.get(timeout=120)
        h = lib.onpu_comm_new(0, 2, 4096)
        mine = (C.c_ubyte * 64)()
        L.check(lib.onpu_comm_ipc_handle(h, mine), "onpu_comm_ipc_handle")
        both = (C.c_ubyte * 128).from_buffer_copy(bytes(mine) + peer_handle)
        L.check(lib.onpu_comm_open(h, both), "onpu_comm_open")
        N, K = 512, 1024
        v, s = O.gen_weights(N, K, seed=1)
        m = DenseMatrix.from_int4(torch.from_numpy(O.pack_baseline(v)).cuda(), torch.from_numpy(s.view(np.int16)).cuda())
        x = torch.from_numpy(O.gen_x(1, K, seed=2)).to(torch.bfloat16).cuda()
        y = torch.empty(1, N, device="cuda")
        L.check(lib.onpu_comm_set_wait(0.2), "onpu_comm_set_wait")
        st = torch.cuda.current_stream().cuda_stream
        L.check(lib.onpu_dense_mv_allreduce_dev(m.h, h, x.data_ptr(), K, 1, y.data_ptr(), None, st), "fused")
        torch.cuda.synchronize()                      # returns: every wait is bounded
        assert lib.onpu_check_device() < 0
        assert "all-reduce timed out" in L.last_error()
        assert lib.onpu_check_device() == 0           # the status was reported once and cleared
        L.check(lib.onpu_comm_set_wait(2.0), "onpu_comm_set_wait")
        ref = O.matmul_xwT(O.gen_x(1, K, seed=2), O.dequant_baseline(v, s))
        y2 = m.mv(x).cpu().numpy()                    # the context still works
        assert np.linalg.norm(y2 - ref) <= 1e-5 * np.linalg.norm(ref)
        assert lib.onpu_check_device() == 0
        assert lib.onpu_comm_set_wait(0.0) < 0 and lib.onpu_comm_set_wait(61.0) < 0
        lib.onpu_comm_free(h)
    finally:
        q_in.put("exit")
        child.join(120)
    assert child.exitcode == 0
