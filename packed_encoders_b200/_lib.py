"""ctypes binding of the C ABI in include/pe_b200_attn.h (``libpe_b200.so``).

The library is the product: there is no Python, Triton, FlashAttention or CPU fallback.
If the shared object is missing or does not load, every entry point raises.
"""

from __future__ import annotations

import ctypes
from functools import lru_cache
from pathlib import Path

from packed_encoders_b200.errors import PackedEncodersError

LIB_PATH = Path(__file__).resolve().parent / "libpe_b200.so"
ABI_VERSION = 4

_p = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64


class PeB200AttnParams(ctypes.Structure):
    """Mirror of ``PeB200AttnParams`` (include/pe_b200_attn.h)."""

    _fields_ = [
        ("q", _p), ("k", _p), ("v", _p), ("out", _p), ("lse", _p),
        ("cu_seqlens_q", _p), ("cu_seqlens_k", _p),
        ("n_seq", _i32), ("total_q", _i32), ("total_k", _i32),
        ("max_seqlen_q", _i32), ("max_seqlen_k", _i32),
        ("heads", _i32), ("kv_heads", _i32), ("head_dim", _i32),
        ("q_stride_token", _i64), ("q_stride_head", _i64),
        ("k_stride_token", _i64), ("k_stride_head", _i64),
        ("v_stride_token", _i64), ("v_stride_head", _i64),
        ("o_stride_token", _i64), ("o_stride_head", _i64),
        ("scale", ctypes.c_float),
        ("window_left", _i32), ("window_right", _i32), ("causal", _i32),
        ("workspace", _p), ("workspace_bytes", ctypes.c_size_t),
        ("gate", _p), ("g_stride_token", _i64), ("g_stride_head", _i64),
        ("rope_cos", _p), ("rope_sin", _p), ("rope_stride_token", _i64),
    ]


class PeB200AttnBwdParams(ctypes.Structure):
    """Mirror of ``PeB200AttnBwdParams`` (include/pe_b200_attn.h)."""

    _fields_ = [
        ("q", _p), ("k", _p), ("v", _p), ("out", _p), ("dout", _p), ("lse", _p),
        ("dq", _p), ("dk", _p), ("dv", _p), ("cu_seqlens", _p),
        ("n_seq", _i32), ("total", _i32), ("max_seqlen", _i32), ("heads", _i32), ("head_dim", _i32),
        ("q_stride_token", _i64), ("q_stride_head", _i64), ("k_stride_token", _i64), ("k_stride_head", _i64),
        ("v_stride_token", _i64), ("v_stride_head", _i64), ("o_stride_token", _i64), ("o_stride_head", _i64),
        ("do_stride_token", _i64), ("do_stride_head", _i64), ("dq_stride_token", _i64), ("dq_stride_head", _i64),
        ("dk_stride_token", _i64), ("dk_stride_head", _i64), ("dv_stride_token", _i64), ("dv_stride_head", _i64),
        ("scale", ctypes.c_float), ("window_left", _i32), ("window_right", _i32), ("causal", _i32),
        ("workspace", _p), ("workspace_bytes", ctypes.c_size_t),
    ]


EXPORTS = (
    "pe_b200_abi_version", "pe_b200_status_string", "pe_b200_last_error_detail", "pe_b200_device_supported",
    "pe_b200_attn_workspace_size", "pe_b200_attn_fwd", "pe_b200_build_schedule", "pe_b200_attn_run",
    "pe_b200_debug_qk", "pe_b200_debug_pv", "pe_b200_rope_qk", "pe_b200_attn_fwd_noalloc",
    "pe_b200_noalloc_error_word", "pe_b200_attn_bwd_workspace_size", "pe_b200_attn_bwd",
)


@lru_cache(maxsize=1)
def lib() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise PackedEncodersError(
            f"{LIB_PATH.name} is not built; run `python -m packed_encoders_b200.build` (nvcc, sm_100a)")
    try:
        so = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:
        raise PackedEncodersError(f"cannot load {LIB_PATH}: {exc}") from exc
    so.pe_b200_abi_version.restype = ctypes.c_int
    so.pe_b200_abi_version.argtypes = []
    if so.pe_b200_abi_version() != ABI_VERSION:
        raise PackedEncodersError("libpe_b200.so ABI version mismatch; rebuild it")
    so.pe_b200_status_string.restype = ctypes.c_char_p
    so.pe_b200_status_string.argtypes = [ctypes.c_int]
    so.pe_b200_last_error_detail.restype = ctypes.c_char_p
    so.pe_b200_last_error_detail.argtypes = []
    so.pe_b200_device_supported.restype = ctypes.c_int
    so.pe_b200_device_supported.argtypes = [ctypes.c_int]
    so.pe_b200_attn_workspace_size.restype = ctypes.c_int
    so.pe_b200_attn_workspace_size.argtypes = [ctypes.POINTER(PeB200AttnParams), ctypes.POINTER(ctypes.c_size_t)]
    for name in ("pe_b200_attn_fwd", "pe_b200_build_schedule", "pe_b200_attn_run"):
        fn = getattr(so, name)
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.POINTER(PeB200AttnParams), _p]
    so.pe_b200_attn_fwd_noalloc.restype = ctypes.c_int
    so.pe_b200_attn_fwd_noalloc.argtypes = [ctypes.POINTER(PeB200AttnParams), _p]
    so.pe_b200_noalloc_error_word.restype = ctypes.c_int
    so.pe_b200_noalloc_error_word.argtypes = [ctypes.POINTER(ctypes.c_int), _p]
    so.pe_b200_attn_bwd_workspace_size.restype = ctypes.c_int
    so.pe_b200_attn_bwd_workspace_size.argtypes = [ctypes.POINTER(PeB200AttnBwdParams), ctypes.POINTER(ctypes.c_size_t)]
    so.pe_b200_attn_bwd.restype = ctypes.c_int
    so.pe_b200_attn_bwd.argtypes = [ctypes.POINTER(PeB200AttnBwdParams), _p]
    so.pe_b200_rope_qk.restype = ctypes.c_int
    so.pe_b200_rope_qk.argtypes = [_p, _p, _i64, _i64, _i64, _i64, _p, _p, _i64, _i32, _i32, _i32, _i32, _i32, _p, _p, _p]
    so.pe_b200_debug_qk.restype = ctypes.c_int
    so.pe_b200_debug_qk.argtypes = [_p, _p, _i64, _i64, ctypes.c_int, ctypes.c_int, ctypes.c_int, _p, _p]
    so.pe_b200_debug_pv.restype = ctypes.c_int
    so.pe_b200_debug_pv.argtypes = [_p, _p, _i64, ctypes.c_int, ctypes.c_int, _p, _p]
    return so


def status_string(status: int) -> str:
    return lib().pe_b200_status_string(int(status)).decode()


def check(status: int, what: str) -> None:
    if status != 0:
        detail = ""
        if status == -7:  # PE_B200_ERR_CUDA: name the CUDA call and its error
            detail = lib().pe_b200_last_error_detail().decode()
            detail = f" [{detail}]" if detail else ""
        raise PackedEncodersError(f"{what} failed: {status_string(status)} (status {status}){detail}")
