"""ctypes binding of librbq.so (the C ABI declared in include/rbq.h).

The product path has no CPU fallback: if the CUDA library is missing or fails to load,
``lib()`` raises immediately with the reason.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "librbq.so")

RBQ_OK = 0
ERRORS = {1: "invalid argument", 2: "CUDA error", 3: "out of device memory", 4: "I/O error",
          5: "wrong call order", 6: "malformed index file"}


class IndexParams(ctypes.Structure):
    _fields_ = [("dim", ctypes.c_int32), ("n_lists", ctypes.c_int32), ("seed", ctypes.c_uint64),
                ("kmeans_n_iters", ctypes.c_int32), ("max_train_points_per_cluster", ctypes.c_int32),
                ("device", ctypes.c_int32), ("shard_rank", ctypes.c_int32), ("shard_count", ctypes.c_int32),
                ("shard_policy", ctypes.c_int32), ("kmeans_kind", ctypes.c_int32), ("raw_store", ctypes.c_int32),
                ("bits_per_dim", ctypes.c_int32)]


class SearchParams(ctypes.Structure):
    _fields_ = [("n_probes", ctypes.c_int32), ("k", ctypes.c_int32), ("rerank", ctypes.c_int32),
                ("prune", ctypes.c_int32), ("probe_split", ctypes.c_int32), ("cand_cap", ctypes.c_int32),
                ("coarse_margin", ctypes.c_int32), ("seeded", ctypes.c_int32), ("query_bits", ctypes.c_int32),
                ("graph", ctypes.c_int32), ("scan_kind", ctypes.c_int32)]


class IndexInfo(ctypes.Structure):
    _fields_ = [("dim", ctypes.c_int32), ("padded_dim", ctypes.c_int32), ("n_lists", ctypes.c_int32),
                ("shard_rank", ctypes.c_int32), ("shard_count", ctypes.c_int32), ("trained", ctypes.c_int32),
                ("n_total", ctypes.c_int64), ("n_local", ctypes.c_int64), ("query_scale", ctypes.c_float),
                ("seed", ctypes.c_uint64), ("device_bytes", ctypes.c_int64), ("shard_policy", ctypes.c_int32),
                ("owners_fixed", ctypes.c_int32), ("kmeans_kind", ctypes.c_int32), ("bits_per_dim", ctypes.c_int32),
                ("ex_scale", ctypes.c_float)]

SHARD_POLICIES = {"round_robin": 0, "balanced": 1}
KMEANS_KINDS = {"balanced": 0, "lloyd": 1}
RAW_STORES = {"device": 0, "host": 1}


# name -> argtypes (all functions return int status unless listed in _RESTYPES)
_P = ctypes.c_void_p
_I32, _I64, _F32, _U64 = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64
SIGNATURES = {
    "rbq_last_error": [],
    "rbq_version": [],
    "rbq_kernel_launches": [],
    "rbq_scan_tile": [],
    "rbq_index_params_default": [ctypes.POINTER(IndexParams)],
    "rbq_search_params_default": [ctypes.POINTER(SearchParams)],
    "rbq_make_rotation": [_I32, _U64, _P],
    "rbq_query_scale": [_I32, _U64, _I32, _P],
    "rbq_list_estimates": [_P, _P, _F32, _F32, _F32, _I32, _P, _P, _P, _I32, _P],
    "rbq_index_create": [ctypes.POINTER(IndexParams), ctypes.POINTER(_P)],
    "rbq_index_free": [_P],
    "rbq_index_info": [_P, ctypes.POINTER(IndexInfo)],
    "rbq_train": [_P, _P, _I64, _P],
    "rbq_set_centroids": [_P, _P, _I32],
    "rbq_build": [_P, _P, _I64, _I32, _P, _P, _P],
    "rbq_add": [_P, _P, _I64, _P, _P],
    "rbq_search": [_P, ctypes.POINTER(SearchParams), _P, _I64, _P, _P, _P],
    "rbq_search_host": [_P, ctypes.POINTER(SearchParams), _P, _I64, _P, _P, _P],
    "rbq_save": [_P, ctypes.c_char_p],
    "rbq_load": [ctypes.c_char_p, _I32, _I32, _I32, ctypes.POINTER(_P)],
    "rbq_import_reference": [ctypes.c_char_p, _I32, _P, _I64, _I32, _I32, _I32, ctypes.POINTER(_P)],
    "rbq_export_reference": [_P, ctypes.c_char_p],
    "rbq_get_rotation": [_P, _P],
    "rbq_get_centroids": [_P, _P, _P],
    "rbq_export_lists": [_P, _P, _P, _P, _P, _P, _P],
    "rbq_export_ex_lists": [_P, _P, _P, _P],
    "rbq_bound_seed_owned": [_P, _P, _P, _P, _P, _I64, _P, _P, _I32, _I32, _I32, _I32, _P, _I32, _P],
    "rbq_scan_lists": [_P, _P, _P, _P, _P, _I64, _P, _P, _I32, _I32, _P, _I32, _P, _P, _P, _I32, _P],
    "rbq_get_list_owners": [_P, _P],
    "rbq_rotate": [_P, _P, _I64, _P, _P],
    "rbq_query_prep": [_P, _P, _I64, _P, _P, _P, _I32, _P],
    "rbq_coarse_scores": [_P, _P, _I64, _P, _I32, _P],
    "rbq_check_errors": [_P],
    "rbq_coarse": [_P, _P, _I64, _I32, _I32, _P, _P, _P],
    "rbq_scan": [_P, _P, _P, _P, _P, _I64, _P, _P, _I32, _I32, _P, _P, _P, _I32, _I32, _I32, _I32, _P, _P, _P, _I32,
                 _P],
    "rbq_bound_seed": [_P, _P, _P, _P, _P, _I64, _P, _P, _I32, _I32, _I32, _I32, _P, _I32, _P],
    "rbq_scan_noalloc": [_P, _P, _P, _P, _P, _I64, _P, _P, _I32, _I32, _P, _I32, _I32, _I32, _I32, _P, _P, _P,
                         _I32, _P],
    "rbq_rerank": [_P, _P, _I64, _P, _I32, _I32, _P, _P, _P],
    "rbq_merge_results": [_P, _P, _I32, _I64, _I32, _P, _P, _P],
    "rbq_pack_results": [_P, _P, _I64, _P, _P],
    "rbq_merge_result_keys": [_P, _I32, _I64, _I32, _P, _P, _P],
    "rbq_debug_fail_alloc": [_I64],
    "rbq_gen_mixture": [_P, _I64, _I32, _I32, _F32, _I32, _I32, _U64, _P],
    "rbq_gen_queries": [_P, _I64, _I32, _P, _I64, _F32, _I32, _U64, _P, _P],
}
_RESTYPES = {"rbq_last_error": ctypes.c_char_p, "rbq_index_params_default": None,
             "rbq_search_params_default": None, "rbq_kernel_launches": ctypes.c_uint64}

_lib = None


def lib() -> ctypes.CDLL:
    """Load librbq.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"neurosamble_b200: CUDA library not built ({LIB_PATH} missing); "
                "run `python -m neurosamble_b200.build_ext`")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = _RESTYPES.get(name, ctypes.c_int)
        _lib = L
    return _lib


def check(status: int) -> None:
    """Raise RuntimeError carrying the library's message for a non-zero status."""
    if status != RBQ_OK:
        msg = lib().rbq_last_error().decode("utf-8", "replace")
        raise RuntimeError(f"rbq error {status} ({ERRORS.get(status, '?')}): {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))


def exported_symbols():
    return list(SIGNATURES)
