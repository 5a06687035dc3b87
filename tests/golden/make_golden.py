"""Generate the golden fixtures in this folder by running the REFERENCE's own Python code.

Run in a container where the reference project is importable (it is not on the GPU box):

    PYTHONPATH=<reference root> python tests/golden/make_golden.py

Every array here comes from the reference's functions (paths relative to its project root):
  geometry.npz  opennpu/native/npu4/model.py:151-190          Mat(N, K, ncols, sym)
  q4nx.npz      opennpu/native/runtime.py:74-82               _requant_q4k
                opennpu/native/npu4/model.py:183-206          Mat.pack (numpy path) ->
                opennpu/native/npu4/gemv_device.py:160-185     pack_block stream order
  q4s.npz       opennpu/native/npu4/model.py:127-147          quant_sym, then Mat.pack (q4s)
  matmul.npz    opennpu/native/reference.py:24-28, :55-57     _wq dequant then h @ W.T (fp32)
  route.npz     opennpu/native/moe_runtime.py:333-341         MoeDecoder._route_with
Inputs are seeded (numpy default_rng) so the script is reproducible.
"""
import os
import sys
import types
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def main():
    import opennpu.native.npu4.model as M
    from opennpu.native import reference as REF
    from opennpu.native.moe_runtime import MoeDecoder
    from opennpu.native.runtime import _requant_q4k
    import torch

    M._CLIB[0], M._CLIB[1] = True, None          # force the numpy packer (no libonpu here)

    # ---- geometry
    shapes = [(4096, 4096), (1024, 4096), (6144, 4096), (12288, 4096), (24576, 4096), (4096, 12288),
              (1536, 2048), (768, 2048), (2048, 768), (17408, 5120), (5120, 17408), (5120, 5120),
              (1024, 5120), (27648, 5120), (5120, 27648), (200, 320), (64, 32), (1, 2048), (100, 96),
              (4096, 2048), (4096, 2080), (130, 16384), (130, 16416)]
    rows = []
    for (N, K) in shapes:
        for nc in (1, 2, 4, 8):
            for sym in (0, 1):
                try:
                    m = M.Mat(N, K, nc, bool(sym))
                    g = (m.R, m.S, m.tiles, m.kc, m.ks, m.rows_col, m.cb, m.nbytes)
                except ValueError:
                    g = (0,) * 8
                rows.append((N, K, nc, sym) + tuple(int(v) for v in g))
    np.savez_compressed(OUT / "geometry.npz", table=np.array(rows, np.int64))

    # ---- q4nx: min/max codec + stream-order pack (numpy path of Mat.pack)
    rng = np.random.default_rng(1234)
    cases = {}
    for name, (N, K, nc) in {"a": (200, 320, 8), "b": (70, 96, 1), "c": (256, 512, 2)}.items():
        W = rng.normal(0, 0.05, size=(N, K)).astype(np.float32)
        q, s, m = _requant_q4k(W)
        packed = M.Mat(N, K, nc, False).pack(W)
        cases.update({f"{name}_W": W, f"{name}_q": q, f"{name}_s": s, f"{name}_m": m,
                      f"{name}_packed": packed, f"{name}_dims": np.array([N, K, nc], np.int64)})
    np.savez_compressed(OUT / "q4nx.npz", **cases)

    # ---- q4s: the numpy symmetric quantiser + pack
    cases = {}
    for name, (N, K, nc) in {"a": (200, 320, 8), "b": (70, 96, 1), "c": (256, 512, 2)}.items():
        W = rng.normal(0, 0.05, size=(N, K)).astype(np.float32)
        q, d = M.quant_sym(W)
        packed = M.Mat(N, K, nc, True).pack(W)
        cases.update({f"{name}_W": W, f"{name}_q": q, f"{name}_d": d, f"{name}_packed": packed,
                      f"{name}_dims": np.array([N, K, nc], np.int64)})
    np.savez_compressed(OUT / "q4s.npz", **cases)

    # ---- the reference's CPU dequantise-then-matmul path
    W = rng.normal(0, 0.05, size=(96, 256)).astype(np.float32)
    x = torch.from_numpy(rng.normal(0, 1, size=(3, 256)).astype(np.float32)).bfloat16().float()
    Wq = REF._wq(W, True)
    y = (x @ Wq.T).numpy()
    np.savez_compressed(OUT / "matmul.npz", W=W, x=x.numpy(), Wq=Wq.numpy(), y=y)

    # ---- the host router (softmax, top-k, sorted ids, renormalised)
    E, H, k, T = 16, 64, 4, 6
    Wr = rng.normal(0, 0.1, size=(E, H)).astype(np.float32)
    h = rng.normal(0, 1, size=(T, H)).astype(np.float32)
    fake = types.SimpleNamespace(routers=[Wr], topk=k, norm_topk=True, E_bo=[list(range(E))])
    ids, ws = [], []
    for t in range(T):
        _, w, top = MoeDecoder._route_with(fake, 0, h[t])
        ids.append(top)
        ws.append(w)
    np.savez_compressed(OUT / "route.npz", Wr=Wr, h=h, k=np.int64(k), ids=np.array(ids, np.int32),
                        w=np.array(ws, np.float32))
    print("wrote", sorted(p.name for p in OUT.glob("*.npz")))


if __name__ == "__main__":
    sys.exit(main())
