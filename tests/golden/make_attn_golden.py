"""Generate tests/golden/attn.npz by running the REFERENCE's own decode attention,
onpu_attn_step / onpu_attn_step_bf16 (llama/ggml-opennpu/onpu_cpu.cpp:173-229), compiled from its
sources into oracle/_ref/libonpu_ref.so (``make -C oracle ref`` in a container that holds the
reference sources):

    python tests/golden/make_attn_golden.py

Each case stores its inputs (the cache as fp32, or as bf16 bits) and the reference's output.
Inputs are seeded (numpy default_rng) so the script is reproducible.
"""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402

OUT = Path(__file__).resolve().parent / "attn.npz"

# name: (Hq, Hkv, D, S, bf16 cache, mask, sinks)
CASES = {
    "gqa4_f32_mask_sinks": (8, 2, 64, 37, False, True, True),
    "gqa4_bf16": (16, 4, 128, 48, True, False, False),
    "mqa5_f32_one_row": (5, 1, 128, 1, False, False, False),
    "mha_bf16_mask_sinks": (4, 4, 64, 70, True, True, True),
    "empty_sinks": (4, 2, 64, 0, False, False, True),
    "all_masked": (2, 1, 64, 9, False, True, False),
}


def main():
    L = O.ref_lib()
    if L is None:
        raise SystemExit("oracle/_ref/libonpu_ref.so is missing: build it with `make -C oracle ref`")
    arrays = {}
    for i, (name, (Hq, Hkv, D, S, bf16, use_mask, use_sinks)) in enumerate(CASES.items()):
        rng = np.random.default_rng(100 + i)
        q = rng.normal(size=(Hq, D)).astype(np.float32)
        K = rng.normal(size=(Hkv, S, D)).astype(np.float32)
        V = rng.normal(size=(Hkv, S, D)).astype(np.float32)
        mask = None
        if use_mask:
            mask = rng.normal(scale=0.5, size=S).astype(np.float32)
            mask[rng.random(S) < 0.2] = -np.inf
            if name == "all_masked":
                mask[:] = -np.inf
        sinks = rng.normal(size=Hq).astype(np.float32) if use_sinks else None
        if bf16:
            K, V = O.f32_to_bf16_bits(K), O.f32_to_bf16_bits(V)
        out = O.attn_step_ref(L, q, K, V, mask, sinks, bf16=bf16)
        arrays[f"{name}.q"] = q
        arrays[f"{name}.K"] = K
        arrays[f"{name}.V"] = V
        arrays[f"{name}.shape"] = np.array([Hq, Hkv, D, S, int(bf16)], np.int64)
        if mask is not None:
            arrays[f"{name}.mask"] = mask
        if sinks is not None:
            arrays[f"{name}.sinks"] = sinks
        arrays[f"{name}.out"] = out
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes, {len(CASES)} cases)")


if __name__ == "__main__":
    main()
