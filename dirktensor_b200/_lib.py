"""ctypes binding of the in-tree CUDA library ``libdirktensor_b200.so``.

The product path has no CPU fallback: if the shared object is missing or does
not load, importing ``dirktensor_b200`` raises.  Build it with
``python -m dirktensor_b200.build``.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# DIRKTENSOR_B200_LIB may point at another build of the same library.
LIB_PATH = os.environ.get("DIRKTENSOR_B200_LIB") or os.path.join(HERE, "libdirktensor_b200.so")

DT_OK = 0
STATUS_NAMES = {
    0: "DT_OK",
    1: "DT_ERR_INVALID_ARGUMENT",
    2: "DT_ERR_CUDA",
    3: "DT_ERR_DEVICE_TIMEOUT",
    4: "DT_ERR_UNSUPPORTED",
    5: "DT_ERR_OUT_OF_MEMORY",
    6: "DT_ERR_IO",
    7: "DT_ERR_NCCL",
    8: "DT_ERR_TIMEOUT",
}


class DTError(RuntimeError):
    """A non-zero status returned through the C ABI."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class dt_attn_weights(ctypes.Structure):
    _fields_ = [
        ("q_proj", ctypes.c_void_p),
        ("k_proj", ctypes.c_void_p),
        ("v_proj", ctypes.c_void_p),
        ("o_proj", ctypes.c_void_p),
        ("q_norm", ctypes.c_void_p),
        ("k_norm", ctypes.c_void_p),
        ("d_model", ctypes.c_int),
        ("n_heads", ctypes.c_int),
        ("eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
    ]


class dt_model_layer_weights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm", "post_attention_norm", "gate_proj", "up_proj",
        "down_proj", "post_feedforward_norm")]


class dt_model_weights(ctypes.Structure):
    _fields_ = [
        ("embed", ctypes.c_void_p),
        ("final_norm", ctypes.c_void_p),
        ("lm_head", ctypes.c_void_p),
        ("layers", ctypes.POINTER(dt_model_layer_weights)),
        ("n_layers", ctypes.c_int),
        ("vocab", ctypes.c_int),
        ("d_model", ctypes.c_int),
        ("n_heads", ctypes.c_int),
        ("hidden", ctypes.c_int),
        ("eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
    ]


_lib = None

_P = ctypes.c_void_p
_I = ctypes.c_int
_LL = ctypes.c_longlong
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> (restype, argtypes); must match include/dirktensor_b200.h
SIGNATURES = {
    "dt_last_error": (ctypes.c_char_p, []),
    "dt_version": (_I, []),
    "dt_check_device_error": (_I, []),
    "dt_selftest_expired_wait": (_I, []),
    "dt_flash_fwd_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "dt_flash_fwd": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I, _P, _SZ, _P]),
    "dt_flash_fwd_host": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I]),
    "dt_gemm_bf16": (_I, [_P, _I, _P, _I, _P, _I, _I, _I, _I, _LL, _P]),
    "dt_flash_bwd_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
    "dt_flash_bwd": (_I, [_P] * 10 + [_I, _I, _I, _I, _F, _I, _P, _SZ, _P]),
    "dt_flash_bwd_host": (_I, [_P] * 10 + [_I, _I, _I, _I, _F, _I]),
    "dt_flash_fwd_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _F, _I, _P]),
    "dt_flash_fwd_bf16_exchange": (_I, [_P, _P, _P, ctypes.POINTER(_P), _I, _I, _LL, _P, _P, _I, _I, _I, _I, _F, _I,
                                        _P]),
    "dt_flash_fwd_qf32_exchange": (_I, [_P, _P, _P, ctypes.POINTER(_P), _I, _I, _LL, _P, _P, _I, _I, _I, _I, _F, _I,
                                        _P]),
    "dt_exchange_barrier": (_I, [ctypes.POINTER(_P), _I, _I, ctypes.c_uint, _P]),
    "dt_ipc_get_handle": (_I, [_P, _P, ctypes.POINTER(_SZ)]),
    "dt_ipc_open": (_I, [_P, _SZ, ctypes.POINTER(_P)]),
    "dt_ipc_close": (_I, [_P, _SZ]),
    "dt_flash_fwd_bf16": (_I, [_P, _P, _P, _P, _I, _LL, _P, _P, _P, _I, _I, _I, _I, _F, _I, _P]),
    "dt_flash_fwd_qf32": (_I, [_P, _P, _P, _P, _I, _LL, _P, _P, _P, _I, _I, _I, _I, _F, _I, _P]),
    "dt_attn_create": (_I, [ctypes.POINTER(dt_attn_weights), _I, ctypes.POINTER(_P)]),
    "dt_attn_create_from_npy": (_I, [ctypes.c_char_p, ctypes.c_uint, _I, ctypes.POINTER(_P)]),
    "dt_attn_forward": (_I, [_P, _P, _I, _I, _P, _P, _P]),
    "dt_attn_forward_host": (_I, [_P, _P, _I, _I, _P, _P]),
    "dt_attn_backward": (_I, [_P, _P, _I, _I, _P, _P]),
    "dt_attn_backward_host": (_I, [_P, _P, _I, _I, _P]),
    "dt_attn_step": (_I, [_P, _F, _P]),
    "dt_attn_zero_grad": (_I, [_P, _P]),
    "dt_attn_get_params_host": (_I, [_P] * 7 + [_I]),
    "dt_attn_destroy": (_I, [_P]),
    "dt_model_create": (_I, [ctypes.POINTER(dt_model_weights), _I, ctypes.POINTER(_P)]),
    "dt_model_create_from_npy": (_I, [ctypes.c_char_p, _I, _I, ctypes.POINTER(_P)]),
    "dt_model_forward": (_I, [_P, _P, _I, _I, _P, _P]),
    "dt_model_forward_host": (_I, [_P, _P, _I, _I, _P]),
    "dt_model_destroy": (_I, [_P]),
    "dt_model_info": (_I, [_P, ctypes.POINTER(_I), ctypes.POINTER(_I), ctypes.POINTER(_I)]),
    "dt_cast_f32_bf16": (_I, [_P, _P, _LL, _P]),
    "dt_cast2_f32_bf16": (_I, [_P, _P, _P, _P, _LL, _P]),
    "dt_gemm_bf16_tn": (_I, [_P, _P, _P, _I, _I, _I, _I, _LL, _P]),
    "dt_gemm_bf16_tn_planar": (_I, [_P, _I, _P, _P, _I, _I, _I, _I, _LL, _P]),
    "dt_qk_norm_rope": (_I, [_P, _P, _P, _LL, _P, _P, _P, _P, _P, _I, _I, _F, _F, _P]),
    "dt_rope_tables": (_I, [_P, _P, _I, _I, _F]),
    "dt_qk_sumsq": (_I, [_P, _P, _LL, _I, _LL, _P, _P]),
    "dt_qk_norm_rope_shard": (_I, [_P, _P, _P, _LL, _P, _P, _P, _I, _P, _P, _P, _I, _I, _F, _F, _P]),
    "dt_comm_unique_id": (_I, [_P]),
    "dt_comm_create": (_I, [_P, _I, _I, _I, _I, ctypes.POINTER(_P)]),
    "dt_comm_abort": (_I, [_P]),
    "dt_comm_destroy": (_I, [_P]),
    "dt_attn_create_sharded": (_I, [ctypes.POINTER(dt_attn_weights), _P, _I, ctypes.POINTER(_P)]),
    "dt_attn_forward_sharded": (_I, [_P, _P, _I, _I, _P, _I, _P, _P]),
    "dt_attn_forward_sharded_host": (_I, [_P, _P, _I, _I, _P, _I, _P]),
    "dt_attn_create_sharded_from_npy": (_I, [ctypes.c_char_p, ctypes.c_uint, _P, _I, ctypes.POINTER(_P)]),
}


def lib():
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} not found: the CUDA library must be built first "
                "(python dirktensor_b200/build.py); there is no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != DT_OK:
        raise DTError(status, lib().dt_last_error().decode(errors="replace"))
