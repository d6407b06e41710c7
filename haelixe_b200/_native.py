"""ctypes binding of libhaelixe_cuda.so (the C ABI in include/haelixe_cuda.h).

This is the Python counterpart of the `extern "C"` block a Rust build of
haelixe declares. There is no fallback: if the library is missing, loading
fails loudly.
"""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libhaelixe_cuda.so")

HX_F32 = 0
HX_BF16 = 1

HX_OK = 0
HX_ERR_INVALID = -1
HX_ERR_UNSUPPORTED = -2
HX_ERR_CUDA = -3
HX_ERR_OOM = -4
HX_ERR_TIMEOUT = -5
HX_ERR_NCCL = -6

HX_GROUP_ID_BYTES = 128
HX_GROUP_REGISTER = 1
HX_GROUP_SYMMETRIC = 2
HX_GROUP_COPY_ENGINE = 4


class HxError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class AttnShape(ctypes.Structure):
    _fields_ = [
        ("B", ctypes.c_int32), ("H", ctypes.c_int32), ("S", ctypes.c_int32), ("D", ctypes.c_int32),
        ("stride_b", ctypes.c_int64), ("stride_h", ctypes.c_int64), ("stride_s", ctypes.c_int64),
    ]


class ArenaStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in
                ("live_bytes", "cached_bytes", "cached_slabs", "cached_bins", "hits", "misses")]


_lib = None

_P = ctypes.c_void_p
class AdamWTensor(ctypes.Structure):
    """hx_adamw_tensor."""
    _fields_ = [("param", ctypes.c_void_p), ("grad", ctypes.c_void_p), ("m", ctypes.c_void_p),
                ("v", ctypes.c_void_p), ("param_lowp", ctypes.c_void_p), ("n", ctypes.c_uint64),
                ("grad_dtype", ctypes.c_int32), ("reserved", ctypes.c_int32)]


_I = ctypes.c_int
_U64 = ctypes.c_uint64
_F = ctypes.c_float
_FP = ctypes.POINTER(ctypes.c_float)
_SHP = ctypes.POINTER(AttnShape)

# name -> (restype, argtypes); mirrors include/haelixe_cuda.h
SIGNATURES = {
    "hx_abi_version": (_I, []),
    "hx_status_string": (ctypes.c_char_p, [_I]),
    "hx_ctx_create": (_I, [_I, ctypes.POINTER(_P)]),
    "hx_ctx_destroy": (_I, [_P]),
    "hx_ctx_device": (_I, [_P, ctypes.POINTER(_I)]),
    "hx_ctx_stream": (_P, [_P]),
    "hx_ctx_set_stream": (_I, [_P, _P]),
    "hx_ctx_use_own_stream": (_I, [_P]),
    "hx_sync": (_I, [_P]),
    "hx_last_error": (_I, [_P, ctypes.c_char_p, ctypes.c_size_t]),
    "hx_bin_size": (_U64, [_U64]),
    "hx_alloc": (_I, [_P, _U64, ctypes.POINTER(_P)]),
    "hx_free": (_I, [_P, _P]),
    "hx_arena_reset": (_I, [_P]),
    "hx_arena_stats_get": (_I, [_P, ctypes.POINTER(ArenaStats)]),
    "hx_copy_h2d": (_I, [_P, _P, _P, _U64]),
    "hx_copy_d2h": (_I, [_P, _P, _P, _U64]),
    "hx_copy_h2d_async": (_I, [_P, _P, _P, _U64]),
    "hx_copy_d2h_async": (_I, [_P, _P, _P, _U64]),
    "hx_host_alloc_pinned": (_I, [_U64, ctypes.POINTER(_P)]),
    "hx_host_free_pinned": (_I, [_P]),
    "hx_flash_attention_fwd": (_I, [_P, _I, _P, _P, _P, _P, _P, _I, _I, _I, _F, _I]),
    "hx_attn_bwd_workspace_size": (_I, [_I, _SHP, ctypes.POINTER(_U64)]),
    "hx_flash_attention_bwd": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _U64,
                                    _I, _I, _I, _F, _I]),
    "hx_flash_attention_bwd_noalloc": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                            _I, _I, _I, _F, _I]),
    "hx_attn_fwd_strided": (_I, [_P, _I, _SHP, _P, _P, _P, _P, _P, _F, _I]),
    "hx_attn_bwd_strided": (_I, [_P, _I, _SHP, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _U64,
                                 _F, _I]),
    "hx_attn_bwd_rope_strided": (_I, [_P, _I, _SHP, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P,
                                      _U64, _F, _I, _F]),
    "hx_linear_fwd": (_I, [_P, _I, _P, _P, _P, _P, _I, _I, _I]),
    "hx_linear_bwd": (_I, [_P, _I, _P, _P, _P, _P, _P, _P, _I, _I, _I]),
    "hx_rmsnorm_fwd": (_I, [_P, _I, _P, _P, _P, _I, _I, _F]),
    "hx_rmsnorm_bwd": (_I, [_P, _I, _P, _P, _P, _P, _P, _I, _I, _F]),
    "hx_linear_residual_fwd": (_I, [_P, _I, _P, _P, _P, _P, _P, _I, _I, _I]),
    "hx_cross_entropy": (_I, [_P, _I, _P, _P, _P, _P, _I, _I]),
    "hx_adamw_step": (_I, [_P, _P, _I, _F, _F, _F, _F, _F, _I]),
    "hx_embedding_fwd": (_I, [_P, _I, _P, _P, _P, _U64, _I, _I]),
    "hx_embedding_bwd": (_I, [_P, _I, _P, _P, _P, _U64, _I, _I]),
    "hx_add": (_I, [_P, _I, _P, _P, _P, _U64]),
    "hx_gelu_fwd": (_I, [_P, _I, _P, _P, _U64]),
    "hx_gelu_bwd": (_I, [_P, _I, _P, _P, _P, _U64]),
    "hx_rope_fwd": (_I, [_P, _I, _SHP, _P, _P, _F]),
    "hx_rope_bwd": (_I, [_P, _I, _SHP, _P, _P, _F]),
    "hx_rope_fwd_qk": (_I, [_P, _I, _SHP, _P, _P, _P, _P, _F]),
    "hx_reassemble_heads": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _I, _I]),
    "hx_torch_malloc": (_P, [ctypes.c_size_t, _I, _P]),
    "hx_torch_free": (None, [_P, ctypes.c_size_t, _I, _P]),
    "hx_torch_arena_context": (_P, [_I]),
    "hx_group_unique_id": (_I, [_P]),
    "hx_group_create_rank": (_I, [_I, _I, _I, _P, _I, _I, ctypes.POINTER(_P)]),
    "hx_group_create": (_I, [_I, ctypes.POINTER(_I), _I, _I, ctypes.POINTER(_P)]),
    "hx_group_destroy": (_I, [_P]),
    "hx_group_abort": (_I, [_P]),
    "hx_group_set_timeout": (_I, [_P, _I]),
    "hx_group_info": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "hx_group_last_error": (_I, [_P, ctypes.c_char_p, _U64]),
    "hx_group_gather_buffer": (_I, [_P, _I, _U64, ctypes.POINTER(_P)]),
    "hx_allgather_heads": (_I, [_P, _I, _P, _I, _P, _P, _I, _I, _I, _I, _I]),
    "hx_group_wait": (_I, [_P, _I, _P]),
    "hx_group_sync": (_I, [_P, _I]),
    "hx_kernel_launches": (_U64, [_P]),
    "hx_last_path": (_I, [_P]),
    "hx_set_force_simt": (_I, [_P, _I]),
    "hx_last_gemm_path": (_I, [_P]),
    "hx_set_gemm_backend": (_I, [_P, _I]),
    "hx_selftest_wait_timeout": (_I, [_P]),
    "hx_arena_set_limit": (_I, [_P, _U64]),
}


def lib():
    """Loads the library (once). Raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m haelixe_b200.build` "
                "(or __graft_entry__.build()); there is no fallback implementation")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error(ctx) -> str:
    buf = ctypes.create_string_buffer(512)
    lib().hx_last_error(ctx, buf, 512)
    return buf.value.decode(errors="replace")


def check(status: int, ctx=None) -> None:
    if status != HX_OK:
        msg = last_error(ctx) if ctx else lib().hx_status_string(status).decode()
        raise HxError(status, msg or lib().hx_status_string(status).decode())
