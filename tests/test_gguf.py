"""GGUF ingest on the CPU: the oracle's restatement of the reference's Q4_K transcode
(llama/ggml-opennpu/ggml-opennpu.cpp:100-143) and of the Q4_0 block, pinned against the weights
the gguf package reads from the same blocks (tests/golden/gguf.npz, tests/golden/make_gguf_golden.py),
and the transcode's choice checked against its definition."""
from pathlib import Path

import numpy as np

from oracle import oracle as O

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "gguf.npz")


def test_q4k_exact_weights_match_gguf():
    assert np.array_equal(O.q4k_exact(GOLD["q4k_blocks"]), GOLD["q4k_weights"])


def test_q4_0_codes_match_gguf():
    q, d = O.q4_0_codes(GOLD["q4_0_blocks"])
    w = (q.astype(np.float32) - 8) * d.view(np.float16).astype(np.float32)[:, None]
    assert np.array_equal(w, GOLD["q4_0_weights"])
    assert q.max() <= 15


def test_q4k_transcode_keeps_codes_and_picks_the_best_bf16_pair():
    blocks = GOLD["q4k_blocks"]
    q, s, m = O.q4k_transcode(blocks)
    exact = GOLD["q4k_weights"].reshape(-1, 8, 32)
    qs = blocks[:, 16:144].reshape(-1, 4, 32)
    for sub in range(8):                               # the codes are the blocks' own nibbles
        want = (qs[:, sub // 2] >> 4) if sub & 1 else (qs[:, sub // 2] & 15)
        assert np.array_equal(q[:, sub], want)
    deq = q.astype(np.float32) * O.bf16_bits_to_f32(s)[..., None] + O.bf16_bits_to_f32(m)[..., None]
    err = np.abs(deq - exact).max() / max(np.abs(exact).max(), 1e-30)
    assert err < 4e-3                                  # bf16 scale and min: ~2^-8 of the block's range


def test_q4k_transcode_is_a_3x3_argmin():
    """For a sample of sub-blocks: recompute the 9 candidates' fp32 errors in the reference's
    operation order and check the chosen pair is the first minimum."""
    blocks = GOLD["q4k_blocks"][:24]
    q, s, m = O.q4k_transcode(blocks)
    for i in range(blocks.shape[0]):
        one = blocks[i:i + 1]
        d = one[:, 0:2].copy().view(np.float16)[:, 0].astype(np.float32)
        dmin = one[:, 2:4].copy().view(np.float16)[:, 0].astype(np.float32)
        for sub in range(8):
            sv, mv = O.q4k_scale_min(one[:, 4:16], sub)
            S = np.float32(d[0] * np.float32(sv[0]))
            M = np.float32(-dmin[0] * np.float32(mv[0]))
            s0, m0 = O.f32_to_bf16_bits(np.array([S]))[0], O.f32_to_bf16_bits(np.array([M]))[0]
            best, pick = np.float32(np.inf), None
            for ds in (-1, 0, 1):
                for dm in (-1, 0, 1):
                    sc = O._bf_step(np.array([s0]), ds)[0] if ds else s0
                    mn = O._bf_step(np.array([m0]), dm)[0] if dm else m0
                    sf = O.bf16_bits_to_f32(np.array([sc]))[0]
                    mf = O.bf16_bits_to_f32(np.array([mn]))[0]
                    e = np.float32(0)
                    for l in range(32):
                        qf = np.float32(q[i, sub, l])
                        x = np.float32(np.float32(np.float32(qf * sf) + mf) - np.float32(np.float32(qf * S) + M))
                        e = np.float32(e + np.float32(x * x))
                    if e < best:
                        best, pick = e, (sc, mn)
            assert (s[i, sub], m[i, sub]) == pick, (i, sub)
