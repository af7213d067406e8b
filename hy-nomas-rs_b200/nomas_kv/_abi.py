"""ctypes declarations of include/nomas_kv.h.

Loads ``libnomas_kv.so`` from this directory (built in-tree by
``hy-nomas-rs_b200/build.py``).  There is no fallback: if the library is
missing or fails to load, every cache operation raises.
"""
from __future__ import annotations

import ctypes as C
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libnomas_kv.so")

NKV_OK = 0
NKV_ERR_GEOMETRY = 1
NKV_ERR_CACHE_STATE = 2
NKV_ERR_INVALID_CONFIG = 3
NKV_ERR_MSG = 4
NKV_ERR_CUDA = 5
NKV_ERR_ARGUMENT = 6

NKV_F32, NKV_BF16, NKV_F16 = 0, 1, 2
NKV_STORAGE_FLOAT, NKV_STORAGE_INT8, NKV_STORAGE_QVG = 0, 1, 2
NKV_SAMPLING_RECENT, NKV_SAMPLING_UNIFORM, NKV_SAMPLING_RECENT_MIX, NKV_SAMPLING_TEMPORAL = 0, 1, 2, 3

NKV_KERNEL_QUANTIZE, NKV_KERNEL_FLOAT_ARCHIVE, NKV_KERNEL_QVG_ENCODE, NKV_KERNEL_GATHER = 0, 1, 2, 3
NKV_KERNEL_SEGMENT_DECODE = 4
NKV_KERNEL_QVG_FIT = 5
NKV_KERNEL_ATTEND = 6
NKV_KERNEL_COUNT = 7
KERNEL_NAMES = ("quantize", "float_archive", "qvg_encode", "gather", "segment_decode", "qvg_fit", "attend")
NKV_NOALLOC_MAX_LAYERS = 64


class nkv_qvg_config(C.Structure):
    _fields_ = [
        ("stages", C.c_int32),
        ("bits_per_stage", C.c_int32),
        ("block_size", C.c_int32),
        ("text_as_int8", C.c_int32),
        ("codebook_seed", C.c_uint64),
    ]


class nkv_cache_config(C.Structure):
    _fields_ = [
        ("storage", C.c_int32),
        ("qvg", nkv_qvg_config),
        ("sampling", C.c_int32),
        ("gamma", C.c_double),
        ("has_capacity", C.c_int32),
        ("capacity", C.c_uint64),
        ("past_frames", C.c_uint64),
        ("phase_swap", C.c_int32),
    ]


class nkv_segment_desc(C.Structure):
    _fields_ = [
        ("segment_index", C.c_uint64),
        ("frame_start", C.c_uint64),
        ("frame_count", C.c_uint64),
        ("image_tokens", C.c_uint64),
        ("text_tokens", C.c_uint64),
        ("action_start", C.c_int64),
    ]


class nkv_segment_layout(C.Structure):
    _fields_ = [
        ("segment_index", C.c_uint64),
        ("video_start", C.c_uint64),
        ("video_end", C.c_uint64),
        ("text_start", C.c_uint64),
        ("text_end", C.c_uint64),
        ("action_start", C.c_int64),
    ]


class nkv_metrics(C.Structure):
    _fields_ = [
        ("archived_segments", C.c_uint64),
        ("archived_bytes", C.c_uint64),
        ("encode_calls", C.c_uint64),
        ("d2h_bytes", C.c_uint64),
        ("h2d_bytes", C.c_uint64),
        ("rebuilds", C.c_uint64),
        ("evicted_tokens", C.c_uint64),
        ("rollbacks", C.c_uint64),
    ]


class nkv_cache_info_t(C.Structure):
    _fields_ = [
        ("valid_len", C.c_uint64),
        ("capacity", C.c_uint64),
        ("n_segments", C.c_uint64),
        ("total_frames", C.c_uint64),
        ("tokens_per_frame", C.c_uint64),
        ("parked", C.c_int32),
        ("storage", C.c_int32),
        ("sampling", C.c_int32),
        ("qvg_fitted", C.c_int32),
    ]


class nkv_kernel_stat(C.Structure):
    _fields_ = [("launches", C.c_uint64), ("total_ms", C.c_double)]


class nkv_staged_layer(C.Structure):
    _fields_ = [("k_codes", C.c_void_p), ("v_codes", C.c_void_p), ("k_scales", C.c_void_p),
                ("v_scales", C.c_void_p), ("status", C.c_void_p)]


class nkv_row_range(C.Structure):
    _fields_ = [("lo", C.c_int64), ("hi", C.c_int64), ("dst", C.c_int64)]


class nkv_kv_project_args(C.Structure):
    _fields_ = [
        ("tokens", C.c_int64), ("heads", C.c_int32), ("head_dim", C.c_int32),
        ("x", C.c_void_p), ("wk", C.c_void_p), ("bk", C.c_void_p), ("wv", C.c_void_p), ("bv", C.c_void_p),
        ("qk_norm", C.c_int32), ("eps", C.c_float), ("k_norm_gain", C.c_void_p),
        ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p),
        ("k_out", C.c_void_p), ("v_out", C.c_void_p),
        ("k_codes", C.c_void_p), ("k_scales", C.c_void_p), ("v_codes", C.c_void_p), ("v_scales", C.c_void_p),
        ("n_ranges", C.c_int32), ("ranges", nkv_row_range * 2),
        ("status", C.c_void_p),
    ]


P = C.c_void_p
U64 = C.c_uint64
I64 = C.c_int64
I32 = C.c_int32

# name -> (restype, argtypes); the same table drives the symbol test.
SIGNATURES = {
    "nkv_last_error": (C.c_char_p, []),
    "nkv_abi_version": (I32, []),
    "nkv_bank_create": (C.c_int, [C.POINTER(nkv_cache_config), I32, I32, I64, I64, I64, I32, I32, P, C.POINTER(P)]),
    "nkv_bank_destroy": (C.c_int, [P]),
    "nkv_bank_commit": (C.c_int, [P, C.POINTER(nkv_segment_desc), I32, C.POINTER(P), C.POINTER(P)]),
    "nkv_bank_rollback": (C.c_int, [P]),
    "nkv_bank_park": (C.c_int, [P]),
    "nkv_bank_unpark": (C.c_int, [P]),
    "nkv_bank_metrics": (C.c_int, [P, C.POINTER(nkv_metrics)]),
    "nkv_bank_synchronize": (C.c_int, [P]),
    "nkv_bank_reserve": (C.c_int, [P, U64, U64]),
    "nkv_bank_segment_bytes": (C.c_int, [P, C.POINTER(nkv_segment_desc), C.POINTER(U64)]),
    "nkv_bank_decode_segment": (C.c_int, [P, U64, C.POINTER(P), C.POINTER(P)]),
    "nkv_bank_attend_history": (C.c_int, [P, I32, P, U64, C.c_float, P, P]),
    "nkv_bank_set_archive_device_limit": (C.c_int, [P, U64]),
    "nkv_bank_archive_usage": (C.c_int, [P, C.POINTER(U64), C.POINTER(U64)]),
    "nkv_bank_commit_decode": (C.c_int, [P, C.POINTER(nkv_segment_desc), I32, C.POINTER(P), C.POINTER(P), C.POINTER(P),
                                         C.POINTER(P)]),
    "nkv_bank_set_timing": (C.c_int, [P, I32]),
    "nkv_bank_kernel_stats": (C.c_int, [P, C.POINTER(nkv_kernel_stat), I32]),
    "nkv_bank_save": (C.c_int, [P, C.c_char_p]),
    "nkv_bank_load": (C.c_int, [P, C.c_char_p]),
    "nkv_bank_stage_segment": (C.c_int, [P, C.POINTER(nkv_segment_desc), C.POINTER(nkv_staged_layer)]),
    "nkv_bank_commit_staged": (C.c_int, [P]),
    "nkv_bank_discard_staged": (C.c_int, [P]),
    "nkv_cache_working_set": (C.c_int, [P, I32, C.POINTER(P), C.POINTER(P), C.POINTER(U64)]),
    "nkv_cache_layout": (C.c_int, [P, I32, C.POINTER(nkv_segment_layout), U64, C.POINTER(U64)]),
    "nkv_cache_info": (C.c_int, [P, I32, C.POINTER(nkv_cache_info_t)]),
    "nkv_cache_metrics": (C.c_int, [P, I32, C.POINTER(nkv_metrics)]),
    "nkv_cache_set_qvg_codebooks": (C.c_int, [P, I32, P]),
    "nkv_cache_get_qvg_codebooks": (C.c_int, [P, I32, P, C.POINTER(I32)]),
    "nkv_cache_export_segment": (C.c_int, [P, I32, U64, P, U64, C.POINTER(U64)]),
    "nkv_frame_indices": (C.c_int, [I32, U64, U64, I32, C.c_double, P, U64, C.POINTER(U64)]),
    "nkv_plan_recent_trim": (C.c_int, [P, U64, U64, U64, P, C.POINTER(U64), P, C.POINTER(U64), C.POINTER(U64), P,
                                       C.POINTER(U64)]),
    "nkv_int8_quantize": (C.c_int, [P, P, I32, U64, I64, P, P, P, P, C.POINTER(C.c_uint32), P]),
    "nkv_int8_dequantize": (C.c_int, [P, P, U64, I64, I32, P, P]),
    "nkv_qvg_encode": (C.c_int, [P, I32, P, I32, U64, I64, I64, U64, I32, I32, I32, P, P, P]),
    "nkv_qvg_decode": (C.c_int, [P, I32, P, P, U64, I64, I64, I32, I32, I32, P, P]),
    "nkv_synth_fill": (C.c_int, [P, I32, U64, I64, I64, U64, U64, P, P, P]),
    "nkv_kv_project": (C.c_int, [C.POINTER(nkv_kv_project_args), P]),
    "nkv_int8_quantize_layers_noalloc": (C.c_int, [C.POINTER(P), C.POINTER(P), I32, I32, U64, I64, C.POINTER(P),
                                                   C.POINTER(P), C.POINTER(P), C.POINTER(P),
                                                   C.POINTER(C.c_uint32), P]),
}

_lib = None


def load(path: str = LIB_PATH):
    """Load the C-ABI library once and declare every entry point."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `python hy-nomas-rs_b200/build.py` "
            "(the cache has no CPU fallback)")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
