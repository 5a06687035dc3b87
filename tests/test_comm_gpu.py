"""The peer-memory all-reduce and the row-parallel GEMV fused with it, on one GPU (a one-rank
group: every word goes to the rank's own buffer through the same code path). The fused call must
give exactly the plain GEMV's outputs (the same sums, sent as 8-byte words and received), fp32
and bf16, over calls that alternate the buffer's two slot sets. The multi-rank behaviour is in
test_multigpu_gpu.py."""
import socket

import numpy as np
import pytest
import torch

from opennpu_b200 import libonpu as L
from opennpu_b200.dense import DenseMatrix
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def peer():
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    torch.distributed.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    from opennpu_b200.comm import PeerAllReduce
    ar = PeerAllReduce(cap_floats=16 * 4096)
    yield ar
    torch.cuda.synchronize()
    ar.close()
    torch.distributed.destroy_process_group()


def test_allreduce_one_rank_is_identity(peer):
    for n in (5120, 37, 4096):
        v = torch.randn(n, device="cuda")
        out = torch.empty_like(v)
        ob = torch.empty(n, device="cuda", dtype=torch.bfloat16)
        peer(v, out=out, out_bf16=ob)
        torch.cuda.synchronize()
        assert torch.equal(out, v)
        assert torch.equal(ob, v.to(torch.bfloat16))
    assert L.load().onpu_check_device() == 0, L.last_error()


@pytest.mark.parametrize("N,K,M,f32", [(4096, 2048, 1, False), (1024, 4096, 3, False), (640, 1536, 16, False),
                                       (5120, 3456, 1, True), (5120, 640, 8, True)])
def test_fused_row_parallel_gemv_matches_plain_gemv(peer, N, K, M, f32):
    """One launch (GEMV epilogue sends, each CTA sums its own rows' words) gives exactly the plain
    GEMV's outputs; bf16 and fp32 activations (the latter: TP = 8 shards of Qwen2.5-32B's down and
    o projections)."""
    from opennpu_b200.comm import PeerAllReduce
    site = PeerAllReduce(cap_floats=M * N)              # one communicator per call site (shape)
    v, s = O.gen_weights(N, K, seed=N + K)
    m = DenseMatrix.from_int4(torch.from_numpy(O.pack_baseline(v)).cuda(), torch.from_numpy(s.view(np.int16)).cuda())
    for call in range(3):                                # both slot sets, then the first again
        x = torch.from_numpy(O.gen_x(M, K, seed=call)).to(torch.bfloat16).cuda()
        if f32:
            x = x.float() + 1e-3 * torch.randn(M, K, device="cuda")
        ref = m.mv(x)
        y = torch.empty(M, N, device="cuda")
        yb = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        site.linear(m, x, out=y, out_bf16=yb)
        torch.cuda.synchronize()
        assert torch.equal(y, ref)
        assert torch.equal(yb, ref.to(torch.bfloat16))
    with pytest.raises(ValueError, match="communicator serves"):       # another activation type: another site
        site.linear(m, x.bfloat16() if f32 else x.float(), out=y)
    assert L.load().onpu_check_device() == 0, L.last_error()
    site.close()


def test_fused_rejects_oversized_and_gateup(peer):
    lib = L.load()
    qk = torch.randint(0, 256, (512, 256), dtype=torch.uint8, device="cuda")
    sc = (torch.rand(512, 16, device="cuda") * 0.02 + 1e-4).half()
    gu = DenseMatrix.from_int4(qk, sc, gateup=True)
    x = torch.zeros(1, 512, dtype=torch.bfloat16, device="cuda")
    y = torch.empty(1, 512, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    assert lib.onpu_dense_mv_allreduce_dev(gu.h, peer.h, x.data_ptr(), 512, 1, y.data_ptr(), 0, st) < 0
    plain = DenseMatrix.from_int4(qk, sc)
    big = torch.zeros(200, 512, dtype=torch.bfloat16, device="cuda")    # more than the buffer holds
    yb = torch.empty(200, 512, device="cuda")
    assert lib.onpu_dense_mv_allreduce_dev(plain.h, peer.h, big.data_ptr(), 512, 200, yb.data_ptr(), 0, st) < 0
