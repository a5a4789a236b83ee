"""ctypes binding of libq8cuda.so (declarations mirror include/q8cuda.h).

The library is built in-tree by ``python -m lama32_mojo_b200.build``.  There
is no fallback: if the shared library is missing or fails to load, importing
the compute entry points raises.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libq8cuda.so")

Q8_OK, Q8_ERR_ARG, Q8_ERR_CUDA, Q8_ERR_OOM, Q8_ERR_KV_FULL, Q8_ERR_IO, Q8_ERR_FORMAT, Q8_ERR_COMM, \
    Q8_ERR_TIMEOUT, Q8_ERR_STATE = range(10)
Q8_F32, Q8_BF16, Q8_F16, Q8_PACKED = range(4)
Q8_ROPE_DEFAULT, Q8_ROPE_LLAMA3 = 0, 1


class q8_config(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("layers", C.c_int32), ("n_heads", C.c_int32),
                ("n_kv", C.c_int32), ("head_dim", C.c_int32), ("inter", C.c_int32),
                ("vocab", C.c_int32), ("eps", C.c_float), ("theta", C.c_double),
                ("rope_factor", C.c_double), ("low_ff", C.c_double), ("high_ff", C.c_double),
                ("orig_ctx", C.c_double), ("rope_type", C.c_int32), ("qk_norm", C.c_int32),
                ("tied", C.c_int32), ("weight_dtype", C.c_int32)]


class Q8Error(RuntimeError):
    """Raised on a non-zero status; ``.status`` holds the code."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"[{status}] {msg}")
        self.status = status


class KVCacheFull(Q8Error):
    pass


_P = C.c_void_p
_I64 = C.c_int64
_I32 = C.c_int
_F = C.c_float

# name -> argtypes (restype is int unless listed in _RESTYPE)
SIGNATURES = {
    "q8_last_error": [_P],
    "q8_status_string": [_I32],
    "q8_version": [],
    "q8_device_status": [],
    "q8_debug_set_device_status": [_I32, _I32],
    "q8op_pack": [_P, _I64, _I64, _P, _P],
    "q8op_dequant": [_P, _I64, _I64, _P, _P],
    "q8op_gemm": [_P, _I32, _I64, _I64, _I64, _P, _I64, _P, _I64, _P],
    "q8op_gemm_noalloc": [_P, _I32, _I64, _I64, _I64, _P, _I64, _P, _I64, _P],
    "q8op_gemm_swiglu": [_P, _I32, _I64, _I64, _I64, _P, _I64, _P, _I64, _P],
    "q8op_gemm_bf16": [_P, _I64, _I64, _I64, _P, _I64, _P, _I64, _P],
    "q8op_embed": [_P, _I64, _I64, _P, _I64, _P, _P],
    "q8op_rmsnorm": [_P, _P, _P, _I64, _I64, _F, _P, _P],
    "q8op_rmsnorm_heads": [_P, _P, _I64, _I64, _F, _P, _P],
    "q8_rope_inv_freq": [C.POINTER(q8_config), _P],
    "q8op_rope_kv_append": [_P, _I64, _I64, _P, _P, _I32, _I32, _I32, _P, _P, _P, _F, _P, _P, _I32,
                            _P, _I32, _P],
    "q8op_attention": [_P, _I64, _I64, _P, _P, _I32, _I32, _I32, _P, _P, _I32, _P, _I32, _P, _I64, _P],
    "q8op_argmax": [_P, _I64, _I64, _I64, _P, _P],
    "q8op_sample": [_P, _I64, _I64, _I64, _F, _F, _P, _P, _P],
    "q8_create": [C.POINTER(q8_config), _I32, _I32, _I32, _I32, _I32, _I32, _P, C.POINTER(_P)],
    "q8_destroy": [_P],
    "q8_nccl_unique_id": [_P],
    "q8_load_tensor": [_P, C.c_char_p, _I32, _I64, _I64, _P, _I32],
    "q8_load_safetensors": [_P, C.c_char_p],
    "q8_forward": [_P, _P, _I32, _I32, _P, _P],
    "q8_decode": [_P, _P, _P, _I32, _P, _P],
    "q8_generate": [_P, _P, _P, _I32, _I32, _P],
    "q8_reset": [_P, _I32],
    "q8_n_cached": [_P, _I32, C.POINTER(_I32)],
    "q8_set_n_cached": [_P, _I32, _I32],
    "q8_stream": [_P, C.POINTER(_P)],
    "q8_set_profiling": [_P, _I32],
    "q8_set_sampling": [_P, _F, _F, C.c_uint64],
    "q8_shard_plan": [C.POINTER(q8_config), _I32, _I32, C.c_char_p] + [C.POINTER(_I64)] * 7 + [C.c_char_p, _I32],
    "q8_inspect_checkpoint": [C.c_char_p, C.c_char_p, C.c_size_t, C.POINTER(_I32)],
    "q8_forward_hidden": [_P, _P, _I32, _I32, _I32, _P],
    "q8_profile": [_P, _I32, C.POINTER(C.c_char_p), C.POINTER(C.c_double), C.POINTER(C.c_double),
                   C.POINTER(_I32), C.POINTER(_I32)],
}
_RESTYPE = {"q8_last_error": C.c_char_p, "q8_status_string": C.c_char_p, "q8_version": C.c_char_p}

_lib = None


def lib() -> C.CDLL:
    """Load libq8cuda.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m lama32_mojo_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = _RESTYPE.get(name, C.c_int)
        _lib = L
    return _lib


def last_error(ctx=None) -> str:
    m = lib().q8_last_error(ctx)
    return m.decode() if m else ""


def check(status: int, ctx=None):
    if status != Q8_OK:
        msg = last_error(ctx)
        if status == Q8_ERR_KV_FULL:
            raise KVCacheFull(status, msg)
        raise Q8Error(status, msg)
