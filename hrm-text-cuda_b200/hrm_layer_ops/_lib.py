"""ctypes binding of the C ABI in include/hrm_ops.h (lib/libhrm_ops.so).

The shared library is the product: there is no Python, PyTorch or CPU
implementation of any operator behind this module.  If the library is missing
the import fails with instructions to build it.
"""

from __future__ import annotations

import ctypes
import os

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG_ROOT, "lib", "libhrm_ops.so")

HRM_OK = 0
HRM_ERR_NULL_POINTER = 1
HRM_ERR_INVALID_SHAPE = 2
HRM_ERR_SIZE_OVERFLOW = 3
HRM_ERR_ALIASING = 4
HRM_ERR_TABLE_RANGE = 5
HRM_ERR_DTYPE = 6
HRM_ERR_SCRATCH_LIMIT = 7
UPLOAD_STATIC_BYTES = 16 * 1024 * 1024  # HRM_UPLOAD_STATIC_BYTES
DTYPES = {"bf16": 0, "f32": 1, "f16": 2}
HRM_ERR_CUDA = 1000

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_f32 = ctypes.c_float

# name -> argument types (every function returns int status).
SIGNATURES = {
    "hrm_additive_inject": [_p, _p, _p, _i64, _p],
    "hrm_rms_norm": [_p, _p, _p, _i64, _i64, _f32, _p],
    "hrm_rms_norm_f32": [_p, _p, _p, _i64, _i64, _f32, _p],
    "hrm_add_rms_norm": [_p, _p, _p, _p, _p, _i64, _i64, _f32, _p],
    "hrm_rope_embed": [_p, _p, _i64, _i64, _i64, _i64, _i64, _f32, _p, _i64, _p],
    "hrm_rope_embed_token_major": [_p, _p, _i64, _i64, _i64, _i64, _i64, _f32, _p, _i64, _p],
    "hrm_rope_table_build": [_p, _i64, _i64, _f32, _p],
    "hrm_swiglu_ffn": [_p, _p, _p, _i64, _p],
    "hrm_embedding_lookup": [_p, _p, _p, _i64, _i64, _i64, _i64, _f32, _p],
    "hrm_embed_rms_norm": [_p, _p, _p, _p, _p, _i64, _i64, _i64, _f32, _f32, _p],
    "hrm_split_gqkv_rope": [_p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _f32, _p, _i64, _i64,
                            _i64, _p],
    "hrm_apply_attn_gate": [_p, _p, _i64, _p],
    "hrm_gated_attn_output": [_p, _p, _p, _i64, _p],
    "hrm_broadcast_vec": [_p, _p, _i64, _i64, _p],
    "hrm_convert_to_bf16": [_p, ctypes.c_int, _p, _i64, _p],
    "hrm_upload_to_bf16": [_p, ctypes.c_int, _p, _i64, _p, _i64, _p],
    "hrm_upload_to_bf16_static": [_p, ctypes.c_int, _p, _i64, _p],
    "hrm_wait_timeouts": [ctypes.POINTER(ctypes.c_uint), ctypes.c_int],
    "hrm_abi_version": [],
}


class HrmError(RuntimeError):
    """A non-zero status from the C ABI (the reference's HrmError)."""

    def __init__(self, op: str, status: int, text: str):
        super().__init__(f"{op}: {text} (status {status})")
        self.op = op
        self.status = status


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `make -C hrm-text-cuda_b200` "
            "(or __graft_entry__.build()); there is no fallback implementation"
        )
    lib = ctypes.CDLL(LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    lib.hrm_status_string.argtypes = [ctypes.c_int]
    lib.hrm_status_string.restype = ctypes.c_char_p
    return lib


LIB = _load()


def check(op: str, status: int) -> None:
    if status != HRM_OK:
        raise HrmError(op, status, LIB.hrm_status_string(status).decode())


def call(name: str, *args) -> None:
    """Calls `name` from the ABI and raises HrmError on a non-zero status."""
    check(name, getattr(LIB, name)(*args))
