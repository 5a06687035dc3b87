"""The ggml op layer's supports predicate (opennpu_supports, llama/ggml-opennpu/ggml-opennpu.cpp:
703-753) on the CPU: which MUL_MAT / MUL_MAT_ID nodes it takes. No GPU is needed to decide."""
import ctypes as C

import numpy as np
import pytest

from opennpu_b200 import libonpu as L

ROW = {L.GGML_F32: lambda K: K * 4, L.GGML_F16: lambda K: K * 2, L.GGML_BF16: lambda K: K * 2,
       L.GGML_Q4_0: lambda K: K // 32 * 18, L.GGML_Q4_K: lambda K: K // 256 * 144}


def tensor(type_, ne, data=1, name=b"blk.0.attn_q.weight", weights=1, nb=None):
    t = L.GgmlTensor()
    t.type, t.weights, t.data, t.name = type_, weights, data, name
    ne = list(ne) + [1] * (4 - len(ne))
    t.ne[:] = ne
    if nb is None:
        rb = ROW[type_](ne[0]) if type_ in ROW else ne[0] * 4
        el = {L.GGML_F32: 4, L.GGML_I32: 4, L.GGML_F16: 2, L.GGML_BF16: 2}.get(type_, 18 if type_ == L.GGML_Q4_0 else 144)
        nb = [el, rb, rb * ne[1], rb * ne[1] * ne[2]]
    t.nb[:] = nb
    return t


def sup(op, w, x=None, dst=None, ids=None, hint=0):
    lib = L.load()
    x = x or tensor(L.GGML_F32, (w.ne[0], 3), weights=0, name=b"x")
    dst = dst or tensor(L.GGML_F32, (w.ne[1], 3), weights=0, name=b"y")
    p = lambda t: C.byref(t) if t is not None else None
    return lib.onpu_ggml_supports(op, p(dst), p(w), p(x), p(ids), hint)


@pytest.mark.parametrize("type_", [L.GGML_F32, L.GGML_F16, L.GGML_BF16, L.GGML_Q4_0, L.GGML_Q4_K])
def test_mul_mat_takes_big_contiguous_weights(type_):
    assert sup(L.GGML_OP_MUL_MAT, tensor(type_, (4096, 1024))) == 1
    assert sup(L.GGML_OP_MUL_MAT, tensor(type_, (1024, 512))) == 0            # below 2^20 parameters


def test_mul_mat_refusals():
    w = tensor(L.GGML_Q4_K, (4096, 1024))
    assert sup(L.GGML_OP_MUL_MAT, w, hint=1) == 0                              # Hadamard-hinted
    assert sup(L.GGML_OP_MUL_MAT, tensor(L.GGML_Q4_K, (4096, 1024), weights=0)) == 0   # not in a weights buffer
    assert sup(L.GGML_OP_MUL_MAT, tensor(L.GGML_Q4_K, (4096, 1024, 2))) == 0    # ne2 != 1
    assert sup(L.GGML_OP_MUL_MAT, tensor(L.GGML_Q4_K, (4000, 1024))) == 0       # Q4_K needs K % 256
    assert sup(L.GGML_OP_MUL_MAT, tensor(L.GGML_F32, (4100, 1024))) == 0        # K % 32
    assert sup(L.GGML_OP_MUL_MAT, tensor(8, (4096, 1024))) == 0                 # Q8_0: not taken
    nb = [144, 16 * 144 + 64, 0, 0]
    nb[2] = nb[1] * 1024
    nb[3] = nb[2]
    assert sup(L.GGML_OP_MUL_MAT, tensor(L.GGML_Q4_K, (4096, 1024), nb=nb)) == 0   # padded rows
    x16 = tensor(L.GGML_F16, (4096, 3), weights=0, name=b"x")
    assert sup(L.GGML_OP_MUL_MAT, w, x=x16) == 0                                # activations must be F32
    assert sup(L.GGML_OP_VIEW, w) == 1


def test_mul_mat_id_takes_quantised_experts():
    ids = tensor(L.GGML_I32, (8, 4), weights=0, name=b"ids")
    w = tensor(L.GGML_Q4_K, (2048, 768, 128), name=b"blk.3.ffn_gate_exps.weight")
    x = tensor(L.GGML_F32, (2048, 1, 4), weights=0, name=b"x")
    dst = tensor(L.GGML_F32, (768, 8, 4), weights=0, name=b"y")
    assert sup(L.GGML_OP_MUL_MAT_ID, w, x=x, dst=dst, ids=ids) == 1
    assert sup(L.GGML_OP_MUL_MAT_ID, tensor(L.GGML_F32, (2048, 768, 128)), x=x, dst=dst, ids=ids) == 0
    assert sup(L.GGML_OP_MUL_MAT_ID, tensor(L.GGML_Q4_K, (256, 256, 8)), x=x, dst=dst, ids=ids) == 0  # < 2^17
    ids_f = tensor(L.GGML_F32, (8, 4), weights=0, name=b"ids")
    assert sup(L.GGML_OP_MUL_MAT_ID, w, x=x, dst=dst, ids=ids_f) == 0            # ids must be I32


def test_cpu_tensors_prefixes_stay_on_the_cpu():
    import subprocess
    import sys
    code = ("import ctypes as C, sys; sys.path.insert(0, '.'); sys.path.insert(0, 'tests');"
            "from opennpu_b200 import libonpu as L; from test_ggml_ops import tensor, sup;"
            "print(sup(L.GGML_OP_MUL_MAT, tensor(L.GGML_Q4_K, (4096, 1024), name=b'blk.0.attn_q.weight')),"
            "      sup(L.GGML_OP_MUL_MAT, tensor(L.GGML_Q4_K, (4096, 1024), name=b'output.weight')))")
    from pathlib import Path
    r = subprocess.run([sys.executable, "-c", code], cwd=Path(__file__).resolve().parents[1], capture_output=True,
                       text=True, env={**__import__("os").environ, "OPENNPU_CPU_TENSORS": "output,token_embd"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == ["1", "0"]
