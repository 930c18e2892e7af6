"""ctypes binding of the C ABI in ``include/qvggt_b200.h``.

The shared library ``libqvggt_b200.so`` is built in-tree by
``python -m qvggt_b200.build``.  There is no fallback: if the library is
missing or a call fails, the error is raised.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libqvggt_b200.so")

vp, i64, i32, u64, f32 = C.c_void_p, C.c_int64, C.c_int32, C.c_uint64, C.c_float
u32p = C.POINTER(C.c_uint32)
i64p = C.POINTER(C.c_int64)

# name -> argtypes (all return int status unless listed in _RESTYPES)
SIGNATURES = {
    "qvggt_version": [],
    "qvggt_last_error": [],
    "qvggt_device_status": [u32p, C.c_int],
    "qvggt_set_wait_timeout_ns": [u64],
    "qvggt_set_gemm_config": [i32],
    "qvggt_launch_count": [],
    "qvggt_w4a16_gemm": [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, vp],
    "qvggt_w4a16_gemm_bf16": [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, vp],
    "qvggt_w4a16_linear_ex": [vp, i64, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i32, i32, vp, i64, vp, vp],
    "qvggt_f16_linear_ex": [vp, i64, vp, vp, vp, i64, i64, i64, i64, i32, vp, i64, vp, vp],
    "qvggt_qkv_rope_linear": [vp, i32, vp, vp, vp, i64, i32, vp, vp, vp, i64, i64, i32, i64, i32, i32, i32, vp, vp,
                              i32, i32, vp, vp, vp, vp, f32, vp],
    "qvggt_w4a16_gemv": [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, vp],
    "qvggt_w4a16_gemv_bf16": [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i32, vp],
    "qvggt_small_linear": [i32, vp, i64, vp, vp, vp, i64, i32, vp, vp, i64, i64, i64, i64, i32, vp, i64, vp, vp],
    "qvggt_small_linear_plan": [i32, i64, i64, i64, C.POINTER(i32)],
    "qvggt_w8a8_gemm": [vp, vp, vp, vp, vp, vp, i64, i64, i64, vp],
    "qvggt_i8_gemm_i32": [vp, vp, vp, i64, i64, i64, vp],
    "qvggt_w8a8_gemm_residual": [vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, vp],
    "qvggt_invoke_quant": [vp, vp, vp, i64, i64, vp],
    "qvggt_layernorm_quant": [vp, vp, vp, vp, vp, i64, i64, f32, i32, vp],
    "qvggt_gelu_quant": [vp, vp, vp, vp, i64, i64, vp],
    "qvggt_layernorm": [vp, vp, vp, vp, i64, i64, f32, vp],
    "qvggt_rope_with_pos": [vp, vp, vp, i64, i64, i64, i64, i64, i64p, i64p, vp],
    "qvggt_qkv_rope2d": [vp, vp, vp, i64, i32, i64, i32, i32, i32, vp, vp, i32, i32, vp, vp, vp, vp, f32, vp],
    "qvggt_attention": [vp, i64, vp, i64, i64, i64, vp, i64, i64, i64, i64, i32, vp],
    "qvggt_attention_ex": [vp, i64, vp, i64, i64, i64, vp, i64, i64, i64, i64, i64, i64, i64, i64, i32, i32, i32, vp,
                           vp, i64, vp],
    "qvggt_attention_plan": [i64, i64, i64, i32, C.POINTER(i32), i64p],
    "qvggt_attention_scratch_bytes": [i64, i64, i32, i32, i64p],
    "qvggt_attention_split_static": [vp, i64, vp, i64, i64, i64, vp, i64, i64, i64, i64, i32, i32, vp],
    "qvggt_attention_small": [vp, i64, vp, i64, i64, i64, vp, i64, i64, i64, i32, vp],
    "qvggt_selftest_wait_timeout": [u64, u32p],
    "qvggt_patchify": [vp, vp, i64, i32, i32, i32, i32, C.POINTER(f32), C.POINTER(f32), vp],
    "qvggt_assemble_tokens": [vp, i64, i64, vp, i32, i32, vp, vp, i64, i32, i32, i64, vp],
    "qvggt_pose_encoding_to_extri_intri": [vp, i64, i32, i32, vp, vp, vp],
    "qvggt_unproject_depth": [vp, i64, i32, i32, vp, vp, vp, vp],
}
_RESTYPES = {"qvggt_last_error": C.c_char_p, "qvggt_launch_count": C.c_uint64}

_lock = threading.Lock()
_lib = None


class QvggtError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, name: str, code: int, msg: str):
        super().__init__(f"{name} failed (code {code}): {msg}")
        self.code = code


def load() -> C.CDLL:
    """Load the library once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} not built; run `python -m qvggt_b200.build`")
            lib = C.CDLL(LIB_PATH)
            for name, args in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = _RESTYPES.get(name, C.c_int)
            _lib = lib
    return _lib


def call(name: str, *args) -> None:
    rc = getattr(load(), name)(*args)
    if rc != 0:
        msg = load().qvggt_last_error().decode(errors="replace")
        raise QvggtError(name, rc, msg)


def launch_count() -> int:
    return int(load().qvggt_launch_count())


def device_status(clear: bool = False) -> int:
    st = C.c_uint32(0)
    call("qvggt_device_status", C.byref(st), 1 if clear else 0)
    return int(st.value)
