"""ctypes binding of the in-tree libonpu.so (the onpu_* C ABI of include/onpu.h).

The argtypes of the reference-compatible part mirror the reference's own binding
(opennpu/native/npu4/model.py:281-335) so the same calls work unchanged. There is no CPU
fallback: ``load()`` raises when the library is missing, and the device paths raise when
``onpu_ok()`` is 0 (no B200).
"""
import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("OPENNPU_LIBONPU", Path(__file__).resolve().parent / "_lib" / "libonpu.so"))

P, I64, I32, F = C.c_void_p, C.c_int64, C.c_int, C.POINTER(C.c_float)
U8P, U16P, I32P, I64P = C.POINTER(C.c_uint8), C.POINTER(C.c_uint16), C.POINTER(C.c_int32), C.POINTER(C.c_int64)

# name -> (restype, argtypes)
SIGNATURES = {
    # ---- reference ABI (onpu_api.cpp / onpu_cpu.cpp)
    "onpu_ok": (I32, []),
    "onpu_batched_ok": (I32, []),
    "onpu_stats": (None, [I64P, C.POINTER(C.c_double)]),
    "onpu_has_shape": (I32, [I32, I32, I32]),
    "onpu_geometry2": (None, [I64, I64, I32, I32, I64P]),
    "onpu_geometry": (None, [I64, I64, I32, I64P]),
    "onpu_dense_new2": (P, [I64, I64, I32]),
    "onpu_dense_new": (P, [I64, I64]),
    "onpu_dense_buf": (U8P, [P]),
    "onpu_dense_bytes": (I64, [P]),
    "onpu_dense_sync": (None, [P]),
    "onpu_dense_mv": (None, [P, F, I64, F]),
    "onpu_dense_free": (None, [P]),
    "onpu_bank_new2": (P, [I64, I64, I64, I32, I32]),
    "onpu_bank_new": (P, [I64, I64, I64, I32]),
    "onpu_bank_buf": (U8P, [P]),
    "onpu_bank_expert_bytes": (I64, [P]),
    "onpu_bank_sync": (None, [P]),
    "onpu_bank_run": (None, [P, F, I32, I64, I32P, I32, F]),
    "onpu_bank_free": (None, [P]),
    "onpu_moe_ffn": (None, [P, P, F, I64, I32P, I32, F, I32, C.c_float, C.c_float, F, F, F]),
    "onpu_moe_act": (None, [F, I64, I64, I32P, F, I32, C.c_float, C.c_float, F]),
    "onpu_moe_sum": (None, [F, I64, I32, I64, I32P, F, F, F]),
    # same argtypes as the reference's binding (npu4/model.py:394-396)
    "onpu_attn_step": (None, [F, I32, I32, F, F, I32, I64, I64, I64, F, F, C.c_float, F]),
    "onpu_attn_step_bf16": (None, [F, I32, I32, F, F, I32, I64, I64, I64, F, F, C.c_float, F]),
    "onpu_ffn_new": (P, [I64, I64, I64, I64, I64, I32]),
    "onpu_ffn_gu": (P, [P]),
    "onpu_ffn_dn": (P, [P]),
    "onpu_ffn_fused": (I32, [P]),
    "onpu_ffn_perm": (None, [P, I32P]),
    "onpu_ffn_run": (I32, [P, F, I32P, I32, F, F]),
    "onpu_ffn_run_many": (I32, [P, F, I64, I32P, I32, F, F]),
    "onpu_ffn_free": (None, [P]),
    "onpu_pack": (I64, [F, I64, I64, I32, I32, U8P, I32]),
    "onpu_quant_dequant": (None, [F, I64, I64, I32, F, I32]),
    # ---- B200 additions
    "onpu_last_error": (C.c_char_p, []),
    "onpu_check_device": (I32, []),
    "onpu_dense_new_int4": (P, [I64, I64, I32]),
    "onpu_dense_load_int4": (I32, [P, P, P, I32, P]),
    "onpu_dense_info": (I32, [P, I64P]),
    "onpu_quantize_dev": (I32, [P, I64, I64, I64, I32, P, P, P, P]),
    "onpu_dense_new_f32_dev": (P, [P, I64, I64, I64, I32, I32, P]),
    "onpu_dense_new_residual_f32_dev": (P, [P, I64, I64, I64, I32, P]),
    "onpu_dense_prepare": (I32, [P, I64]),
    "onpu_ggml_supports": (I32, [I32, P, P, P, P, I32]),
    "onpu_ggml_new": (P, []),
    "onpu_ggml_note": (None, [P, I32, P, P, P]),
    "onpu_ggml_compute": (I32, [P, I32, P, P, P, P]),
    "onpu_ggml_stats": (None, [P, I64P]),
    "onpu_ggml_free": (None, [P]),
    "onpu_gguf_codes_dev": (I32, [I32, P, I64, I64, P, P, P, P]),
    "onpu_dense_new_gguf": (P, [I64, I64, I32, P, I32, I32, P]),
    "onpu_bank_new_gguf": (P, [I64, I64, I64, I32, P, I32, I32, P]),
    "onpu_dense_mv_dev": (I32, [P, P, I64, I64, P, I64, I32, P]),
    "onpu_dense_mv_f32_dev": (I32, [P, P, I64, I64, P, I64, I32, P]),
    "onpu_dense_max_f32_rows": (I32, [P]),
    "onpu_dense_mv_dev_noalloc": (I32, [P, P, I64, I64, P, I64, I32, P]),
    "onpu_dense_mm_dev": (I32, [P, P, I64, I64, P, I64, I32, P]),
    "onpu_dense_unpack_dev": (I32, [P, P, P, P, P]),
    "onpu_attn_step_dev": (I32, [P, I32, I32, P, P, I32, I64, I64, I64, P, P, C.c_float, P, I32, P]),
    "onpu_layout_version": (I32, []),
    "onpu_dense_export": (I64, [P, P, I64]),
    "onpu_dense_import": (P, [P, I64]),
    "onpu_bank_export": (I64, [P, P, I64]),
    "onpu_bank_import": (P, [P, I64]),
    "onpu_ffn_export": (I64, [P, P, I64]),
    "onpu_ffn_import": (P, [P, I64]),
    "onpu_route_dev": (I32, [P, I64, I64, P, I64, I64, I32, I32, P, P, P, P]),
    "onpu_bank_new_int4": (P, [I64, I64, I64, I32]),
    "onpu_bank_load_int4": (I32, [P, P, P, I32, P]),
    "onpu_ffn_new_int4": (P, [I64, I64, I64, I64, I64]),
    "onpu_moe_ffn_dev": (I32, [P, P, I64, I64, P, P, I32, P, I64, P]),
    "onpu_moe_ffn_dev_ep": (I32, [P, P, I64, I64, P, P, I32, I64, P, I64, P]),
    "onpu_moe_layer_dev": (I32, [P, P, P, I64, I64, I32, I32, P, P, P, I64, P]),
    "onpu_moe_set_fused": (I32, [I32]),
    "onpu_comm_new": (P, [I32, I32, I64]),
    "onpu_comm_ipc_handle": (I32, [P, P]),
    "onpu_comm_open": (I32, [P, P]),
    "onpu_comm_allreduce": (I32, [P, P, P, P, I64, P]),
    "onpu_comm_free": (None, [P]),
    "onpu_comm_set_wait": (I32, [C.c_double]),
    "onpu_dense_mv_allreduce_dev": (I32, [P, P, P, I64, I64, P, P, P]),
    "onpu_dense_mv_allreduce_f32_dev": (I32, [P, P, P, I64, I64, P, P, P]),
    "onpu_chain_new": (P, []),
    "onpu_chain_add": (I32, [P, P, P, I64, I64, P, I64, I32, I32]),
    "onpu_chain_info": (I32, [P, I64P]),
    "onpu_chain_link_dep": (I32, [P, I32]),
    "onpu_chain_prepare": (I32, [P]),
    "onpu_chain_run": (I32, [P, P]),
    "onpu_chain_trace": (I32, [P, P]),
    "onpu_chain_free": (None, [P]),
    "onpu_gemv_trace": (I32, [P, I64]),
}

_LIB = None


class OnpuError(RuntimeError):
    pass


def load():
    """The library handle with every signature bound; raises if libonpu.so was not built."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise OnpuError(f"{LIB_PATH} is missing: build it with `python -m opennpu_b200.build`")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def last_error():
    e = load().onpu_last_error()
    return e.decode() if e else None


BLOB_MAGIC = b"ONPUB2GL"
BLOB_DENSE, BLOB_BANK, BLOB_FFN = 1, 2, 3
BLOB_GATEUP, BLOB_RESIDUAL = 1, 2


def blob_sections(blob):
    """The matrix headers of a weight blob (onpu_*_export): (kind, [{N, K, E, fmt, flags, bytes}]).
    Reads only the headers; the library validates the whole blob on import."""
    import struct
    mv = memoryview(blob).cast("B")
    if len(mv) < 64 or bytes(mv[:8]) != BLOB_MAGIC:
        raise OnpuError("not a weight blob")
    version, kind, nmats = struct.unpack_from("<III", mv, 8)
    mats, off = [], 64
    for _ in range(nmats):
        if len(mv) < off + 64:
            raise OnpuError("weight blob truncated")
        N, K, E, fmt, flags, nbytes = struct.unpack_from("<qqqiIq", mv, off)
        mats.append(dict(N=N, K=K, E=E, fmt=fmt, flags=flags, bytes=nbytes, version=version))
        off += 64 + (nbytes + 63) // 64 * 64
    return kind, mats


def export_blob(fn, h, what):
    """Run an onpu_*_export entry twice (size, then contents) -> the blob as a uint8 numpy array."""
    import numpy as np
    n = fn(h, None, 0)
    check(n, what)
    buf = np.empty(n, dtype=np.uint8)
    check(fn(h, buf.ctypes.data, n), what)
    return buf


def as_blob(blob):
    """bytes / bytearray / memoryview / numpy -> a contiguous uint8 numpy array (no copy when possible)."""
    import numpy as np
    if isinstance(blob, np.ndarray):
        return np.ascontiguousarray(blob.view(np.uint8).reshape(-1))
    return np.frombuffer(blob, dtype=np.uint8)


def check(rc, what="libonpu call"):
    """Raise OnpuError with the library's message when rc < 0 (or rc is a NULL handle)."""
    if rc is None or (isinstance(rc, int) and rc < 0):
        raise OnpuError(f"{what}: {last_error() or 'failed'}")
    return rc


def require_device():
    lib = load()
    if not lib.onpu_ok():
        raise OnpuError("libonpu: no usable B200 (onpu_ok() == 0); there is no CPU fallback")
    return lib


def fp(a):
    return a.ctypes.data_as(F)


def i32p(a):
    return a.ctypes.data_as(I32P)


class GgmlTensor(C.Structure):
    """onpu_ggml_tensor: the ggml_tensor fields the ggml op layer reads (include/onpu.h)."""
    _fields_ = [("type", C.c_int32), ("weights", C.c_int32), ("ne", C.c_int64 * 4), ("nb", C.c_int64 * 4),
                ("data", C.c_void_p), ("name", C.c_char_p)]


GGML_OP_VIEW, GGML_OP_MUL_MAT, GGML_OP_MUL_MAT_ID = 0, 1, 2
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_K, GGML_I32, GGML_BF16 = 0, 1, 2, 12, 26, 30
