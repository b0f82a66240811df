"""ctypes binding of ``libmh3_b200.so`` (the C ABI declared in include/mh3_b200.h).

The library is built in-tree by ``python -m minimaxh3_b200.build``.  There is
no fallback: if the library is missing or fails to load, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmh3_b200.so")
_lock = threading.Lock()
_lib = None

MH3_OK = 0
MH3_ERR_INVALID = -1
MH3_ERR_UNSUPPORTED = -2
MH3_ERR_DRIVER = -3
MH3_ERR_TOO_LARGE = -4
MH3_DTYPE_BF16 = 0
MH3_DTYPE_F16 = 1
MH3_DTYPE_E4M3 = 2
MH3_DTYPE_F32 = 3
MH3_DEVERR_WAIT_TIMEOUT = 1
MH3_PEER_HANDLE_BYTES = 64
MH3_TEST_STALL_PRODUCER = 1

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_u64 = ctypes.c_uint64
c_f32 = ctypes.c_float
c_ptr = ctypes.c_void_p


class AttnArgs(ctypes.Structure):
    """``mh3_attn_args`` (include/mh3_b200.h)."""

    _fields_ = [
        ("batch", c_i32), ("heads", c_i32), ("seqlen_q", c_i32), ("seqlen_k", c_i32),
        ("head_dim", c_i32), ("out_dtype", c_i32), ("v_dtype", c_i32), ("test_flags", c_i32),
        ("q8", c_ptr), ("q_stride_b", c_i64), ("q_stride_h", c_i64), ("q_stride_s", c_i64),
        ("k8", c_ptr), ("k_stride_b", c_i64), ("k_stride_h", c_i64), ("k_stride_s", c_i64),
        ("v8", c_ptr), ("v_stride_b", c_i64), ("v_stride_h", c_i64), ("v_stride_s", c_i64),
        ("out", c_ptr), ("o_stride_b", c_i64), ("o_stride_h", c_i64), ("o_stride_s", c_i64),
        ("scale_q", c_ptr), ("sq_stride_b", c_i64), ("sq_stride_h", c_i64), ("sq_stride_blk", c_i64),
        ("scale_k", c_ptr), ("sk_stride_b", c_i64), ("sk_stride_h", c_i64), ("sk_stride_blk", c_i64),
        ("scale_v", c_ptr), ("sv_stride_b", c_i64), ("sv_stride_h", c_i64), ("sv_stride_d", c_i64),
        ("logit_scale_log2", c_f32), ("max_seqlen_q", c_i32),
        ("cu_seqlens_q", c_ptr), ("cu_seqlens_k", c_ptr),
        ("total_q", c_i64), ("total_k", c_i64),
        ("key_bias2", c_ptr), ("key_bias2_stride_b", c_i64),
        ("err", c_ptr), ("timeout_ns", c_u64), ("kv_len", c_ptr),
    ]


class QkvQuantArgs(ctypes.Structure):
    """``mh3_qkv_quant_args`` (include/mh3_b200.h)."""

    _fields_ = [
        ("batch", c_i32), ("heads", c_i32), ("seqlen_q", c_i32), ("seqlen_k", c_i32),
        ("head_dim", c_i32), ("in_dtype", c_i32),
        ("q", c_ptr), ("q_stride_b", c_i64), ("q_stride_h", c_i64), ("q_stride_s", c_i64),
        ("k", c_ptr), ("k_stride_b", c_i64), ("k_stride_h", c_i64), ("k_stride_s", c_i64),
        ("v", c_ptr), ("v_stride_b", c_i64), ("v_stride_h", c_i64), ("v_stride_s", c_i64),
        ("q_premul", c_f32), ("v_out_dtype", c_i32),
        ("q8", c_ptr), ("k8", c_ptr), ("v8", c_ptr),
        ("scale_q", c_ptr), ("scale_k", c_ptr), ("scale_v", c_ptr), ("k_mean", c_ptr),
        ("workspace", c_ptr),
    ]


class GemmArgs(ctypes.Structure):
    """``mh3_gemm_args`` (include/mh3_b200.h)."""

    _fields_ = [
        ("M", c_i64), ("N", c_i64), ("K", c_i64), ("R", c_i64),
        ("ab_dtype", c_i32), ("row_scale_inv", c_i32),
        ("a", c_ptr), ("lda", c_i64), ("b", c_ptr), ("ldb", c_i64),
        ("row_scale", c_ptr), ("col_scale", c_ptr), ("bias", c_ptr),
        ("a2", c_ptr), ("lda2", c_i64), ("b2", c_ptr), ("ldb2", c_i64),
        ("out", c_ptr), ("ldo", c_i64), ("err", c_ptr), ("timeout_ns", c_u64),
        ("test_flags", c_i32), ("reserved1", c_i32),
    ]


# name -> (restype, argtypes)
_SIGNATURES = {
    "mh3_abi_version": (c_i32, []),
    "mh3_last_error": (ctypes.c_char_p, []),
    "mh3_device_error_word": (c_ptr, []),
    "mh3_fp8_attention_fwd": (c_i32, [ctypes.POINTER(AttnArgs), c_ptr]),
    "mh3_key_bias": (c_i32, [c_ptr, c_i64, c_ptr, c_i64, c_i64, c_i64, c_ptr, c_i64, c_ptr, c_ptr]),
    "mh3_qkv_workspace_bytes": (c_u64, [c_i32, c_i32, c_i32, c_i32]),
    "mh3_quantize_qkv": (c_i32, [ctypes.POINTER(QkvQuantArgs), c_ptr]),
    "mh3_quantize_qkv_noalloc": (c_i32, [ctypes.POINTER(QkvQuantArgs), c_ptr]),
    "mh3_quantize_rows": (c_i32, [c_ptr, c_i64, c_i32, c_i64, c_i64, c_ptr, c_ptr, c_ptr]),
    "mh3_widen_e4m3_to_f16": (c_i32, [c_ptr, c_ptr, c_i64, c_ptr]),
    "mh3_scaled_gemm": (c_i32, [ctypes.POINTER(GemmArgs), c_ptr]),
    "mh3_absmax_bh": (c_i32, [c_ptr, c_i32, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_i32,
                              c_ptr, c_ptr]),
    "mh3_quantize_bh": (c_i32, [c_ptr, c_i32, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_i32,
                                c_ptr, c_i32, c_ptr, c_ptr]),
    "mh3_absmax_seg": (c_i32, [c_ptr, c_i32, c_i64, c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_i32, c_ptr, c_i32,
                               c_ptr, c_ptr]),
    "mh3_quantize_seg": (c_i32, [c_ptr, c_i32, c_i64, c_i64, c_i64, c_i64, c_i64, c_i32, c_i32, c_i32, c_ptr, c_i32,
                                 c_ptr, c_i32, c_ptr, c_ptr]),
    "mh3_copy_rows": (c_i32, [c_ptr, c_i64, c_ptr, c_i64, c_i64, c_i64, c_ptr]),
    "mh3_peer_alloc": (c_i32, [c_i64, c_ptr]),
    "mh3_peer_free": (c_i32, [c_ptr]),
    "mh3_peer_handle": (c_i32, [c_ptr, c_ptr]),
    "mh3_peer_open": (c_i32, [c_ptr, c_ptr]),
    "mh3_peer_close": (c_i32, [c_ptr]),
    "mh3_step_diff_workspace_bytes": (c_u64, []),
    "mh3_step_diff": (c_i32, [c_ptr, c_ptr, c_i32, c_i64, c_i32, c_ptr, c_ptr, c_ptr]),
}

EXPORTED = tuple(_SIGNATURES)


class Mh3Error(RuntimeError):
    """A libmh3_b200 call returned a non-zero status."""


def lib_path() -> str:
    return _LIB_PATH


def load():
    """Load the library (once).  Raises if it is missing: there is no fallback."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(_LIB_PATH):
            raise Mh3Error(
                f"{_LIB_PATH} is missing; build it with `python -m minimaxh3_b200.build` "
                "(the CUDA path has no CPU fallback)")
        lib = ctypes.CDLL(_LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != MH3_OK:
        msg = load().mh3_last_error().decode(errors="replace")
        if rc < 0:
            raise ValueError(f"{what}: {msg} (status {rc})")
        raise Mh3Error(f"{what}: {msg} (CUDA error {rc})")
