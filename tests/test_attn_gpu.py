"""Decode attention on the GPU (attn.cu) against the reference: the golden vectors of its own
onpu_attn_step(_bf16) and the float64 oracle at model sizes. The GPU sums in fp32 in another
order than the reference, so the bound is fp32 rounding: 1e-5 of the largest output (max-abs),
NaN exactly where the reference gives NaN."""
import ctypes as C

import numpy as np
import pytest
import torch

from opennpu_b200 import libonpu as L
from opennpu_b200.attn import attn_step
from oracle import oracle as O
from tests.test_attn_oracle import assert_attn_close, golden_cases, widen

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _dev(c):
    dt = torch.bfloat16 if c["bf16"] else torch.float32
    if c["bf16"]:
        K = torch.from_numpy(c["K"].view(np.int16)).view(torch.bfloat16)
        V = torch.from_numpy(c["V"].view(np.int16)).view(torch.bfloat16)
    else:
        K, V = torch.from_numpy(c["K"]), torch.from_numpy(c["V"])
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t(c["q"]), K.to(dt).cuda(), V.to(dt).cuda(), t(c["mask"]), t(c["sinks"])


@pytest.mark.parametrize("c", golden_cases(), ids=lambda c: c["name"])
def test_device_matches_reference_golden(c):
    q, K, V, m, sk = _dev(c)
    y = attn_step(q, K, V, m, sk)
    torch.cuda.synchronize()
    assert_attn_close(y.cpu().numpy(), c["out"], TOL)


@pytest.mark.parametrize("c", golden_cases(), ids=lambda c: c["name"])
def test_host_abi_matches_reference_golden(c):
    """onpu_attn_step / _bf16 with host pointers, called as the reference's binding calls it."""
    lib = L.require_device()
    q, K, V = c["q"], np.ascontiguousarray(c["K"]), np.ascontiguousarray(c["V"])
    Hq, D = q.shape
    Hkv, S, _ = K.shape
    out = np.full((Hq, D), 7.0, np.float32)
    f = lib.onpu_attn_step_bf16 if c["bf16"] else lib.onpu_attn_step
    fp = lambda a: None if a is None else np.ascontiguousarray(a).ctypes.data_as(L.F)
    f(fp(q), Hq, D, K.ctypes.data_as(L.F), V.ctypes.data_as(L.F), Hkv, S, S * D, D, fp(c["mask"]),
      fp(c["sinks"]), D ** -0.5, fp(out))
    assert L.last_error() is None
    assert_attn_close(out, c["out"], TOL)


@pytest.mark.parametrize("Hq,Hkv,D,S,bf16,sinks", [
    (32, 8, 128, 4096, True, False),     # Qwen3-8B layer, 4k context
    (40, 8, 128, 1000, True, False),     # Qwen2.5-32B: 5 query heads per kv head
    (64, 8, 64, 777, False, True),       # gpt-oss-like: sinks, fp32 cache
    (16, 16, 256, 65, True, False),      # D = 256, no GQA
    (32, 2, 128, 20000, True, False),    # 16 query heads per kv head, long context
])
def test_device_matches_oracle_at_model_sizes(Hq, Hkv, D, S, bf16, sinks):
    g = torch.Generator(device="cuda").manual_seed(S + Hq)
    q = torch.randn(Hq, D, device="cuda", generator=g)
    dt = torch.bfloat16 if bf16 else torch.float32
    K = torch.randn(Hkv, S, D, device="cuda", generator=g).to(dt)
    V = torch.randn(Hkv, S, D, device="cuda", generator=g).to(dt)
    mask = torch.where(torch.rand(S, device="cuda", generator=g) < 0.05, float("-inf"), 0.0)
    sk = torch.randn(Hq, device="cuda", generator=g) if sinks else None
    y = attn_step(q, K, V, mask, sk)
    ref = O.attn_step(q.cpu().numpy(), K.float().cpu().numpy(), V.float().cpu().numpy(), mask.cpu().numpy(),
                      None if sk is None else sk.cpu().numpy())
    assert_attn_close(y.cpu().numpy(), ref, TOL)


def test_strided_cache_slice():
    """A static cache [Hkv, Smax, D] read for its first S rows: head stride Smax * D."""
    Hq, Hkv, D, Smax, S = 8, 2, 128, 512, 300
    g = torch.Generator(device="cuda").manual_seed(1)
    cache_k = torch.randn(Hkv, Smax, D, device="cuda", generator=g).to(torch.bfloat16)
    cache_v = torch.randn(Hkv, Smax, D, device="cuda", generator=g).to(torch.bfloat16)
    cache_k[:, S:] = float("nan")                       # rows past S must never be read
    cache_v[:, S:] = float("nan")
    q = torch.randn(Hq, D, device="cuda", generator=g)
    y = attn_step(q, cache_k[:, :S], cache_v[:, :S])
    ref = O.attn_step(q.cpu().numpy(), cache_k[:, :S].float().cpu().numpy(), cache_v[:, :S].float().cpu().numpy())
    assert_attn_close(y.cpu().numpy(), ref, TOL)
    assert torch.equal(y, attn_step(q, cache_k[:, :S].contiguous(), cache_v[:, :S].contiguous()))


def test_repeat_calls_are_deterministic():
    g = torch.Generator(device="cuda").manual_seed(2)
    q = torch.randn(32, 128, device="cuda", generator=g)
    K = torch.randn(8, 3000, 128, device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn(8, 3000, 128, device="cuda", generator=g).to(torch.bfloat16)
    a = attn_step(q, K, V)
    assert torch.equal(a, attn_step(q, K, V))


def test_rejects_unsupported_shapes():
    q = torch.zeros(6, 64, device="cuda")
    K = torch.zeros(4, 8, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(L.OnpuError):                    # Hq % Hkv != 0
        attn_step(q, K, K)
    q = torch.zeros(4, 20, device="cuda")
    K = torch.zeros(2, 8, 20, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(L.OnpuError):                    # 20 bf16 = 40 bytes: not whole 16-byte chunks
        attn_step(q, K, K)
    q = torch.zeros(34, 64, device="cuda")
    K = torch.zeros(2, 8, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(L.OnpuError):                    # 17 query heads per kv head
        attn_step(q, K, K)
    torch.cuda.synchronize()
    assert L.load().onpu_check_device() == 0, L.last_error()


@pytest.mark.parametrize("Hq,Hkv,D,S", [(64, 8, 64, 3000), (28, 4, 128, 2000), (8, 8, 64, 257)])
def test_tensor_core_form_masks_and_sinks(Hq, Hkv, D, S):
    """The bf16 tensor-core form at its limits (8 and 7 query heads per kv head, D 64 and 128) with
    sinks and masks whose -inf runs blank whole splits, and a cache masked everywhere (NaN without
    sinks, as the reference; zeros with them)."""
    g = torch.Generator(device="cuda").manual_seed(Hq * S)
    q = torch.randn(Hq, D, device="cuda", generator=g)
    K = torch.randn(Hkv, S, D, device="cuda", generator=g).to(torch.bfloat16)
    V = torch.randn(Hkv, S, D, device="cuda", generator=g).to(torch.bfloat16)
    sk = torch.randn(Hq, device="cuda", generator=g)
    mask = torch.zeros(S, device="cuda")
    mask[: S // 2] = float("-inf")                       # the first half of the rows: many whole splits
    mask[S // 2 + 3::7] = float("-inf")
    Kf, Vf = K.float().cpu().numpy(), V.float().cpu().numpy()
    for m, s in ((mask, sk), (mask, None), (None, sk)):
        y = attn_step(q, K, V, m, s)
        ref = O.attn_step(q.cpu().numpy(), Kf, Vf, None if m is None else m.cpu().numpy(),
                          None if s is None else s.cpu().numpy())
        assert_attn_close(y.cpu().numpy(), ref, TOL)
    full = torch.full((S,), float("-inf"), device="cuda")
    assert torch.isnan(attn_step(q, K, V, full)).all()
    assert torch.equal(attn_step(q, K, V, full, sk), torch.zeros(Hq, D, device="cuda"))
    torch.cuda.synchronize()
    assert L.load().onpu_check_device() == 0, L.last_error()
