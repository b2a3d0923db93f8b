"""ctypes binding of ``libsas.so`` (the C ABI declared in ``include/sas.h``).

The product path has no CPU fallback: if the library is missing, importing a
compute entry point raises with the build command to run.
"""

from __future__ import annotations

import ctypes as C
import os
from typing import Optional

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libsas.so")

# ---- status codes / enums (sas.h) ----
SAS_OK = 0
ERRORS = {1: "SAS_ERR_INVALID", 2: "SAS_ERR_UNSUPPORTED", 3: "SAS_ERR_CUDA",
          4: "SAS_ERR_SCHEDULE", 5: "SAS_ERR_WORKSPACE", 6: "SAS_ERR_DEVICE"}
LAYOUTS = {"BSND": 0, "TND": 1, "BSH": 2, "BNSD": 3, "PA_ND": 4}
DTYPE_BF16, DTYPE_FP16 = 0, 1
SCENARIO_SWA, SCENARIO_CFA, SCENARIO_SCFA = 1, 2, 3
PHASE_ATTN, PHASE_COMBINE, PHASE_ALL = 1, 2, 3
SAS_META_SIZE = 1024
SAS_NOALLOC_SCRATCH_BYTES = 16 << 20
SAS_AIC_CORE_NUM = 36
SAS_AIV_CORE_NUM = 72
SAS_FA_METADATA_SIZE = 8
SAS_FD_METADATA_SIZE = 8

_i64p = C.POINTER(C.c_int64)
_i32p = C.POINTER(C.c_int32)


class SasMetaParams(C.Structure):
    _fields_ = [
        ("num_heads_q", C.c_int64), ("num_heads_kv", C.c_int64), ("head_dim", C.c_int64),
        ("cu_seqlens_q", _i64p), ("n_cu_seqlens_q", C.c_int64),
        ("cu_seqlens_ori_kv", _i64p), ("n_cu_seqlens_ori_kv", C.c_int64),
        ("cu_seqlens_cmp_kv", _i64p), ("n_cu_seqlens_cmp_kv", C.c_int64),
        ("seqused_q", _i64p), ("n_seqused_q", C.c_int64),
        ("seqused_kv", _i64p), ("n_seqused_kv", C.c_int64),
        ("batch_size", C.c_int64), ("max_seqlen_q", C.c_int64), ("max_seqlen_kv", C.c_int64),
        ("ori_topk", C.c_int64), ("cmp_topk", C.c_int64), ("cmp_ratio", C.c_int64),
        ("ori_mask_mode", C.c_int32), ("cmp_mask_mode", C.c_int32),
        ("ori_win_left", C.c_int64), ("ori_win_right", C.c_int64),
        ("layout_q", C.c_int32), ("layout_kv", C.c_int32),
        ("has_ori_kv", C.c_int32), ("has_cmp_kv", C.c_int32),
        ("aic_core_num", C.c_int64), ("aiv_core_num", C.c_int64),
    ]


class SasProblem(C.Structure):
    _fields_ = [
        ("batch", C.c_int32), ("layout_q", C.c_int32), ("max_q_len", C.c_int32),
        ("total_tokens", C.c_int32), ("q_start", _i32p), ("q_len", _i32p), ("kv_len", _i32p),
        ("num_heads", C.c_int32), ("scenario", C.c_int32), ("ori_win_left", C.c_int32),
        ("cmp_ratio", C.c_int32), ("topk", C.c_int32),
    ]


class SasFwdParams(C.Structure):
    _fields_ = [
        ("q", C.c_void_p), ("ori_kv", C.c_void_p), ("ori_block_table", C.c_void_p),
        ("cmp_kv", C.c_void_p), ("cmp_block_table", C.c_void_p), ("cmp_indices", C.c_void_p),
        ("sinks", C.c_void_p), ("out", C.c_void_p), ("lse", C.c_void_p), ("err", C.c_void_p),
        ("head_dim", C.c_int32), ("head_dim_v", C.c_int32), ("dtype", C.c_int32),
        ("softmax_scale", C.c_float),
        ("ori_block_size", C.c_int32), ("ori_num_blocks", C.c_int32),
        ("ori_table_len", C.c_int32),
        ("cmp_block_size", C.c_int32), ("cmp_num_blocks", C.c_int32),
        ("cmp_table_len", C.c_int32),
        ("num_sms", C.c_int32), ("trace", C.c_void_p),
        ("slot_dump", C.c_void_p), ("slot_dump_cap", C.c_int32),
    ]


class SasPlanInfo(C.Structure):
    _fields_ = [
        ("num_rows", C.c_int32), ("num_workers", C.c_int32), ("head_groups", C.c_int32),
        ("num_split_rows", C.c_int32), ("num_partials", C.c_int32),
        ("total_tiles", C.c_int64), ("plan_ints", C.c_int64), ("split_off", C.c_int64),
        ("actq_off", C.c_int64), ("actkv_off", C.c_int64),
    ]


# Exported symbols and their prototypes (must match include/sas.h).
PROTOTYPES = {
    "sas_metadata": (C.c_int, [C.POINTER(SasMetaParams), _i32p, C.c_size_t]),
    "sas_fwd_workspace_size": (C.c_int, [C.POINTER(SasProblem), C.c_int32,
                                         C.POINTER(C.c_size_t)]),
    "sas_fwd": (C.c_int, [C.POINTER(SasProblem), C.POINTER(SasFwdParams), C.c_void_p,
                          C.c_size_t, C.c_void_p]),
    "sas_fwd_prepare": (C.c_int, [C.POINTER(SasProblem), C.POINTER(SasFwdParams), C.c_void_p,
                                  C.c_size_t, C.c_void_p, C.POINTER(SasPlanInfo)]),
    "sas_fwd_execute": (C.c_int, [C.POINTER(SasProblem), C.POINTER(SasFwdParams),
                                  C.POINTER(SasPlanInfo), C.c_void_p, C.c_size_t, C.c_void_p,
                                  C.c_int32]),
    "sas_fwd_workspace_size_device": (C.c_int, [C.POINTER(SasProblem), C.c_int32,
                                                C.POINTER(C.c_size_t)]),
    "sas_fwd_prepare_device": (C.c_int, [C.POINTER(SasProblem), C.POINTER(SasFwdParams),
                                         C.c_void_p, C.c_size_t, C.c_void_p,
                                         C.POINTER(SasPlanInfo)]),
    "sas_fwd_noalloc": (C.c_int, [C.POINTER(SasProblem), C.POINTER(SasFwdParams),
                                  C.c_void_p]),
    "sas_kv_append": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
                                C.c_int32, C.c_void_p, C.c_void_p]),
    "sas_combine": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p,
                              C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                              C.c_void_p, C.c_void_p]),
    "sas_plan_size": (C.c_int, [C.POINTER(SasProblem), C.c_int32, C.POINTER(SasPlanInfo)]),
    "sas_plan": (C.c_int, [C.POINTER(SasProblem), C.c_int32, _i32p, C.c_int64,
                           C.POINTER(SasPlanInfo)]),
    "sas_error_string": (C.c_char_p, [C.c_int]),
    "sas_version": (C.c_char_p, []),
    "sas_device_sm_count": (C.c_int32, []),
}

_LIB: Optional[C.CDLL] = None


class SasError(RuntimeError):
    """A libsas call returned a non-zero status."""

    def __init__(self, fn: str, code: int):
        self.code = code
        msg = lib().sas_error_string(code).decode() if _LIB is not None else ""
        super().__init__(f"{fn} failed: {ERRORS.get(code, code)} ({msg})")


def lib() -> C.CDLL:
    """Load libsas.so once; raise if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with "
                "`python -m sparse_attn_sharedkv_b200.build` (nvcc, sm_100a). "
                "There is no CPU fallback.")
        handle = C.CDLL(LIB_PATH)
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(fn: str, code: int) -> None:
    if code != SAS_OK:
        raise SasError(fn, code)
