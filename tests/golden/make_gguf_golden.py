"""Generate tests/golden/gguf.npz: seeded GGUF Q4_0 and Q4_K blocks and the weights the installed
gguf package (gguf-py, the reader the reference calls at opennpu/native/gguf_ckpt.py:55-56)
dequantises them to. The reference's own Q4_K transcode (llama/ggml-opennpu/ggml-opennpu.cpp:
100-143) needs the ggml headers, absent here, so its inputs are pinned through gguf's reading of
the same blocks: the oracle's exact weights must equal these, and its transcoded codes must be the
blocks' own nibbles.

    python tests/golden/make_gguf_golden.py
"""
from pathlib import Path

import numpy as np


def q4k_blocks(rng, n):
    b = rng.integers(0, 256, size=(n, 144), dtype=np.uint8)
    d = (np.abs(rng.normal(0, 0.005, n)) + 1e-4).astype(np.float16)
    dmin = np.abs(rng.normal(0, 0.005, n)).astype(np.float16)
    d[:4] = [0.0, 6e-8, 1e-3, 0.25]                  # zero, fp16-subnormal, small, large super-block scales
    dmin[:4] = [0.0, 1e-3, 0.0, 6e-8]
    b[:, 0:2] = d.view(np.uint8).reshape(n, 2)
    b[:, 2:4] = dmin.view(np.uint8).reshape(n, 2)
    b[4, 4:16] = 0                                   # every 6-bit scale and min zero
    b[5, 4:16] = 255                                 # every one 63
    return b


def q4_0_blocks(rng, n):
    b = rng.integers(0, 256, size=(n, 18), dtype=np.uint8)
    d = (np.abs(rng.normal(0, 0.02, n)) + 1e-4).astype(np.float16)
    d[:2] = [0.0, -0.01]
    b[:, 0:2] = d.view(np.uint8).reshape(n, 2)
    return b


def main():
    import gguf
    rng = np.random.default_rng(2024)
    k = q4k_blocks(rng, 96)
    z = q4_0_blocks(rng, 96)
    wk = gguf.quants.dequantize(k.reshape(-1), gguf.GGMLQuantizationType.Q4_K).reshape(96, 256).astype(np.float32)
    wz = gguf.quants.dequantize(z.reshape(-1), gguf.GGMLQuantizationType.Q4_0).reshape(96, 32).astype(np.float32)
    out = Path(__file__).resolve().parent / "gguf.npz"
    np.savez_compressed(out, q4k_blocks=k, q4k_weights=wk, q4_0_blocks=z, q4_0_weights=wz)
    print(out)


if __name__ == "__main__":
    main()
