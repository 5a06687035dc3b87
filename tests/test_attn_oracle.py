"""The decode-attention oracle (oracle.attn_step, float64) pinned to the reference's own
onpu_attn_step / onpu_attn_step_bf16: against the committed golden vectors
(tests/golden/make_attn_golden.py) and, where oracle/_ref was built, against the live library on
further shapes. The reference sums in fp32, so the bound is fp32 rounding: 1e-6 of the largest
output."""
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden" / "attn.npz"


def golden_cases():
    g = np.load(GOLDEN)
    names = sorted({k.split(".")[0] for k in g.files})
    out = []
    for n in names:
        Hq, Hkv, D, S, bf16 = (int(v) for v in g[f"{n}.shape"])
        K, V = g[f"{n}.K"], g[f"{n}.V"]
        out.append(dict(name=n, q=g[f"{n}.q"], K=K, V=V, bf16=bool(bf16),
                        mask=g[f"{n}.mask"] if f"{n}.mask" in g.files else None,
                        sinks=g[f"{n}.sinks"] if f"{n}.sinks" in g.files else None, out=g[f"{n}.out"]))
    return out


def widen(c):
    return (O.bf16_bits_to_f32(c["K"]), O.bf16_bits_to_f32(c["V"])) if c["bf16"] else (c["K"], c["V"])


def assert_attn_close(y, ref, tol=1e-6):
    y, ref = np.asarray(y, np.float64), np.asarray(ref, np.float64)
    assert y.shape == ref.shape
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    ok = ~np.isnan(ref)
    if ok.any():
        assert np.abs(y[ok] - ref[ok]).max() <= tol * max(1.0, np.abs(ref[ok]).max())


@pytest.mark.parametrize("c", golden_cases(), ids=lambda c: c["name"])
def test_oracle_matches_reference_golden(c):
    K, V = widen(c)
    assert_attn_close(O.attn_step(c["q"], K, V, c["mask"], c["sinks"]), c["out"])


def test_golden_edge_cases_are_what_the_reference_gives():
    cases = {c["name"]: c for c in golden_cases()}
    assert np.array_equal(cases["empty_sinks"]["out"], np.zeros_like(cases["empty_sinks"]["out"]))
    assert np.isnan(cases["all_masked"]["out"]).all()


REF = O.ref_lib()


@pytest.mark.skipif(REF is None, reason="oracle/_ref not built (needs the reference sources)")
@pytest.mark.parametrize("Hq,Hkv,D,S,bf16", [(40, 8, 128, 200, True), (64, 8, 64, 150, False), (6, 3, 96, 33, True)])
def test_oracle_matches_live_reference(Hq, Hkv, D, S, bf16):
    rng = np.random.default_rng(Hq + S)
    q = rng.normal(size=(Hq, D)).astype(np.float32)
    K = rng.normal(size=(Hkv, S, D)).astype(np.float32)
    V = rng.normal(size=(Hkv, S, D)).astype(np.float32)
    mask = np.where(rng.random(S) < 0.1, -np.inf, 0.0).astype(np.float32)
    sinks = rng.normal(size=Hq).astype(np.float32)
    if bf16:
        Kb, Vb = O.f32_to_bf16_bits(K), O.f32_to_bf16_bits(V)
        ref = O.attn_step_ref(REF, q, Kb, Vb, mask, sinks, scale=0.1, bf16=True)
        K, V = O.bf16_bits_to_f32(Kb), O.bf16_bits_to_f32(Vb)
    else:
        ref = O.attn_step_ref(REF, q, K, V, mask, sinks, scale=0.1)
    assert_attn_close(O.attn_step(q, K, V, mask, sinks, scale=0.1), ref)
