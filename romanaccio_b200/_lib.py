"""ctypes binding of the C ABI declared in include/w8a8.h (libw8a8.so, built in-tree).

Loading fails loudly when the shared library is missing: there is no CPU fallback for the
W8A8 path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libw8a8.so"

# w8a8_status (mirrors es_status_t, es_runtime.h:24-35)
SUCCESS = 0
ERR_INVALID_ARG = -1
ERR_NO_MEMORY = -2
ERR_DEVICE_BUSY = -3
ERR_HARDWARE_FAULT = -4
ERR_NOT_INITIALIZED = -5
ERR_NOT_SUPPORTED = -6
ERR_IO = -7
ERR_CHECKSUM_MISMATCH = -8
ERR_TIMEOUT = -9
ERR_CUDA = -10
ERR_PEER_TIMEOUT = -11

DTYPE_FP16, DTYPE_INT8, DTYPE_INT16 = 0, 1, 2
ACT_STATIC, ACT_DYNTOK = 0, 1
OUT_ACC_I32, OUT_QUANT, OUT_F32, OUT_F32_ACC = 0, 1, 2, 3
TOPK_MAX = 64
PATH_AUTO, PATH_GEMV, PATH_TENSOR, PATH_TENSOR_PAIR = 0, 1, 2, 3
TC_MIN_TOKENS = 16


class ScaleInfo(C.Structure):
    _fields_ = [
        ("out_dtype", C.c_int32),
        ("in_thresh", C.c_float),
        ("in_step", C.c_float),
        ("out_thresh", C.c_float),
        ("out_step", C.c_float),
        ("in_inv_smooth", C.c_void_p),
        ("out_step_chan", C.c_void_p),
    ]


class LinearDesc(C.Structure):
    _fields_ = [
        ("K", C.c_int32),
        ("N", C.c_int32),
        ("weights", C.c_void_p),
        ("weights_ld", C.c_int64),
        ("quant_m", C.c_void_p),
        ("trunc", C.c_int32),
        ("acc_step", C.c_void_p),
        ("scale", ScaleInfo),
    ]


class MoeDesc(C.Structure):
    _fields_ = [
        ("hidden", C.c_int32),
        ("inter", C.c_int32),
        ("n_routed", C.c_int32),
        ("n_shared", C.c_int32),
        ("top_k", C.c_int32),
        ("norm_topk_prob", C.c_int32),
        ("routed_scaling", C.c_float),
        ("max_tokens", C.c_int32),
        ("gate_w", C.c_void_p),
        ("gate_bias", C.c_void_p),
        ("gu_weights", C.c_void_p),
        ("gu_quant_m", C.c_void_p),
        ("gu_out_step_chan", C.c_void_p),
        ("gu_inv_smooth", C.c_void_p),
        ("gu_in_thresh", C.c_void_p),
        ("gu_trunc", C.c_int32),
        ("dn_weights", C.c_void_p),
        ("dn_quant_m", C.c_void_p),
        ("dn_out_step_chan", C.c_void_p),
        ("dn_inv_smooth", C.c_void_p),
        ("dn_in_step", C.c_void_p),
        ("dn_trunc", C.c_int32),
        ("dn_out_dtype", C.c_int32),
    ]


class SamplerParams(C.Structure):
    """w8a8_sampler_params (mirrors eswin::SamplerParams, sampler.hpp:10-19)."""
    _fields_ = [
        ("temperature", C.c_float),
        ("top_k", C.c_int32),
        ("top_p", C.c_float),
        ("min_p", C.c_float),
        ("repeat_penalty", C.c_float),
        ("repeat_window", C.c_int32),
        ("max_consecutive_duplicates", C.c_int32),
        ("seed", C.c_uint32),
    ]


class ChainStep(C.Structure):
    _fields_ = [
        ("linear", C.c_void_p),
        ("x_dev", C.c_void_p),
        ("ldx", C.c_int64),
        ("act_mode", C.c_int32),
        ("out_mode", C.c_int32),
        ("y_dev", C.c_void_p),
        ("ldy", C.c_int64),
        ("ratio_dev", C.c_void_p),
        ("topk_k", C.c_int32),
        ("row_offset", C.c_int32),
        ("topk_val_dev", C.c_void_p),
        ("topk_idx_dev", C.c_void_p),
        ("emb_norm_dev", C.c_void_p),
        ("norm_eps", C.c_float),
    ]


# name -> (restype, argtypes); every symbol include/w8a8.h declares.
_P, _I32, _I64, _SZ = C.c_void_p, C.c_int32, C.c_int64, C.c_size_t
SIGNATURES = {
    "w8a8_status_to_string": (C.c_char_p, [C.c_int]),
    "w8a8_last_error": (C.c_char_p, []),
    "w8a8_version": (C.c_char_p, []),
    "w8a8_ctx_create": (C.c_int, [C.c_int, C.POINTER(_P)]),
    "w8a8_ctx_destroy": (None, [_P]),
    "w8a8_ctx_sm_count": (C.c_int, [_P]),
    "w8a8_ctx_device": (C.c_int, [_P]),
    "w8a8_ctx_check": (C.c_int, [_P]),
    "w8a8_linear_create": (C.c_int, [_P, C.POINTER(LinearDesc), C.POINTER(_P)]),
    "w8a8_linear_destroy": (None, [_P]),
    "w8a8_linear_device_bytes": (_SZ, [_P]),
    "w8a8_linear_set_path": (C.c_int, [_P, _I32]),
    "w8a8_linear_reserve": (C.c_int, [_P, _I32, _I32, _P]),
    "w8a8_linear_set_input_norm": (C.c_int, [_P, _P, C.c_float]),
    "w8a8_linear_set_trace": (C.c_int, [_P, _P]),
    "w8a8_pack_input": (C.c_int, [_P, _P, _I64, _I32, _I32, _P, _I64, _P, _P]),
    "w8a8_linear_forward_q": (C.c_int, [_P, _P, _I64, _I32, _I32, _P, _I32, _P, _I64, _P]),
    "w8a8_unpack_output": (C.c_int, [_P, _P, _I64, _I32, _I32, _P, _P, _I64, _P]),
    "w8a8_linear_forward": (C.c_int, [_P, _P, _I64, _I32, _I32, _I32, _P, _I64, _P, _P]),
    "w8a8_linear_forward_topk": (
        C.c_int, [_P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _P, _P, _P, _I64, _P]),
    "w8a8_topk_merge": (C.c_int, [_P, _P, _P, _I32, _I32, _I32, _I64, _I64, _I32, _P, _P, _P, _P]),
    "w8a8_lmhead_create": (C.c_int, [C.POINTER(_P), _I32, _I32, _I32, _P, _I64, _P, C.c_float,
                                     _I32, _I32, C.POINTER(_P)]),
    "w8a8_lmhead_forward": (C.c_int, [_P, _P, _I32, _I32, _P, _P, _P, _P]),
    "w8a8_lmhead_destroy": (None, [_P]),
    "w8a8_lmhead_shards": (_I32, [_P]),
    "w8a8_lmhead_set_trace": (C.c_int, [_P, _P, C.POINTER(_P)]),
    "w8a8_lmhead_rank_create": (C.c_int, [_P, _I32, _I32, _I32, _I32, _P, _I64, _P, C.c_float,
                                          _I32, _I32, C.POINTER(_P)]),
    "w8a8_lmhead_rank_export": (C.c_int, [_P, _P]),
    "w8a8_lmhead_rank_connect": (C.c_int, [_P, _P]),
    "w8a8_lmhead_rank_connect_local": (C.c_int, [C.POINTER(_P), _I32]),
    "w8a8_lmhead_rank_forward": (C.c_int, [_P, _P, _I32, _I32, _P, _P, _P, _P]),
    "w8a8_lmhead_rank_destroy": (None, [_P]),
    "w8a8_lmhead_rank_set_input_norm": (C.c_int, [_P, _P, C.c_float]),
    "w8a8_lmhead_set_input_norm": (C.c_int, [_P, _P, C.c_float]),
    "w8a8_emb_norm_pack": (C.c_int, [_P, _P, _I64, _I32, _I32, _P, C.c_float, _P, _I64, _P]),
    "w8a8_linear16_create": (C.c_int, [_P, _I32, _I32, _P, _I64, _P, _I32, _P, _I32,
                                       C.POINTER(_P)]),
    "w8a8_linear16_forward": (C.c_int, [_P, _P, _I64, _I32, _I32, _P, _I64, _P]),
    "w8a8_linear16_destroy": (None, [_P]),
    "w8a8_lmhead_rank_shard_range": (_I32, [_P, C.POINTER(_I32), C.POINTER(_I32)]),
    "w8a8_moe_create": (C.c_int, [_P, C.POINTER(MoeDesc), C.POINTER(_P)]),
    "w8a8_moe_destroy": (None, [_P]),
    "w8a8_moe_route": (C.c_int, [_P, _P, _I64, _I32, _P, _P, _P]),
    "w8a8_moe_forward": (C.c_int, [_P, _P, _I64, _I32, _P, _I64, _P]),
    "w8a8_moe_ep_create": (C.c_int, [_P, _I32, _I32, _I32, C.POINTER(_P)]),
    "w8a8_moe_ep_export": (C.c_int, [_P, _P]),
    "w8a8_moe_ep_connect": (C.c_int, [_P, _P]),
    "w8a8_moe_ep_connect_local": (C.c_int, [C.POINTER(_P), _I32]),
    "w8a8_moe_ep_forward": (C.c_int, [_P, _P, _I64, _I32, _P, _I64, _P]),
    "w8a8_moe_ep_destroy": (None, [_P]),
    "w8a8_moe_views": (C.c_int, [_P, C.POINTER(_P), C.POINTER(_P), C.POINTER(_P), C.POINTER(_P),
                                 C.POINTER(_P)]),
    "w8a8_chain_create": (C.c_int, [_P, C.POINTER(ChainStep), _I32, _I32, C.POINTER(_P)]),
    "w8a8_chain_forward": (C.c_int, [_P, _P]),
    "w8a8_chain_destroy": (None, [_P]),
    "w8a8_chain_barriers": (_I32, [_P]),
    "w8a8_chain_grid": (_I32, [_P]),
    "w8a8_chain_set_trace": (C.c_int, [_P, _P]),
    "w8a8_rmsnorm_pack_dyntok": (C.c_int, [_P, _P, _I64, _I32, _I32, _P, _P, C.c_float,
                                         C.c_float, _P, _I64, _P, _P, _I64, _P]),
    "w8a8_post_op_ffn_pack": (C.c_int, [_P, _P, _I64, _P, _P, _I64, _I32, _I32, _P, C.c_float,
                                        _P, _I64, _P, _I64, _P]),
    "w8a8_sampler_create": (C.c_int, [C.POINTER(SamplerParams), C.POINTER(_P)]),
    "w8a8_sampler_destroy": (None, [_P]),
    "w8a8_sampler_accept": (C.c_int, [_P, _I32]),
    "w8a8_sampler_reset": (C.c_int, [_P]),
    "w8a8_sampler_sample": (C.c_int, [_P, _P, _P, _I32, _I32, _P]),
    "w8a8_lmhead_topk_noalloc": (
        C.c_int, [_P, _I64, _I32, _I32, _P, C.c_float, _P, _I64, _I32, _I32, _I32, _P, _P, _P]),
}


class W8A8Error(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(what)


_lib = None


def load() -> C.CDLL:
    """Loads libw8a8.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python -m romanaccio_b200.build` "
            "(the W8A8 path has no CPU fallback)")
    lib = C.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, what: str = "") -> None:
    if status != SUCCESS:
        lib = load()
        msg = lib.w8a8_status_to_string(status).decode()
        detail = lib.w8a8_last_error().decode()
        raise W8A8Error(status, f"{what}: {msg} ({status}): {detail}")
