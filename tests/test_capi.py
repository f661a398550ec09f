"""The C-ABI library (librbq.so): loads, exports every symbol include/rbq.h declares, and its
host-only logic (constants, error paths, file parsing) behaves without a GPU."""
import ctypes
import os
import re

import numpy as np
import pytest

from neurosamble_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rbq.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rbq_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "rbq_search" in syms and "rbq_build" in syms and "rbq_last_error" in syms
    assert len(syms) >= 25


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name


def test_binding_covers_header():
    assert set(declared_symbols()) == set(_lib.exported_symbols())


def test_version():
    assert _lib.lib().rbq_version() == 1


def test_host_rotation_matches_oracle(oracle):
    for dp, seed in ((32, 7), (128, 3), (256, 7)):
        P = np.empty((dp, dp), np.float32)
        _lib.call("rbq_make_rotation", dp, seed, P.ctypes.data_as(ctypes.c_void_p))
        assert np.array_equal(P.view(np.uint32), oracle.make_rotation(dp, seed).view(np.uint32))
        t = ctypes.c_float()
        _lib.call("rbq_query_scale", dp, seed, 3, ctypes.byref(t))
        assert np.float32(t.value).view(np.uint32) == np.float32(oracle.query_scale(dp, seed)).view(np.uint32)


def test_invalid_arguments_return_status():
    P = np.empty((4, 4), np.float32)
    st = _lib.lib().rbq_make_rotation(4, 1, P.ctypes.data_as(ctypes.c_void_p))
    assert st == 1
    assert b"multiple of 32" in _lib.lib().rbq_last_error()
    with pytest.raises(RuntimeError, match="invalid argument"):
        _lib.call("rbq_make_rotation", 33, 1, P.ctypes.data_as(ctypes.c_void_p))


def test_load_rejects_missing_and_malformed_files(tmp_path):
    h = ctypes.c_void_p()
    st = _lib.lib().rbq_load(str(tmp_path / "nope.rbq").encode(), 0, -1, 0, ctypes.byref(h))
    assert st == 4 and not h.value
    bad = tmp_path / "bad.rbq"
    bad.write_bytes(b"NOTANIDX" + b"\0" * 64)
    st = _lib.lib().rbq_load(str(bad).encode(), 0, -1, 0, ctypes.byref(h))
    assert st == 6 and b"not an RBQB200" in _lib.lib().rbq_last_error()
    trunc = tmp_path / "trunc.rbq"
    trunc.write_bytes(b"RBQB200\0" + b"\x01\0\0\0")
    st = _lib.lib().rbq_load(str(trunc).encode(), 0, -1, 0, ctypes.byref(h))
    assert st == 6 and b"truncated" in _lib.lib().rbq_last_error()


def test_null_arguments_are_rejected():
    L = _lib.lib()
    assert L.rbq_index_create(None, None) == 1
    assert L.rbq_search(None, None, None, 0, None, None, None) == 1
    assert L.rbq_index_free(None) == 0


def test_product_has_no_oracle_dependency():
    """The product package never imports or links the oracle."""
    pkg = os.path.join(ROOT, "neurosamble_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".h")):
                text = open(os.path.join(dirpath, f), errors="ignore").read()
                assert "oracle" not in re.sub(r"(#|//).*", "", text).lower() or f == "build_ext.py", f


def test_parameter_defaults():
    """Host-only: the defaults a C caller gets (reference defaults where one exists)."""
    L = _lib.lib()
    ip = _lib.IndexParams()
    L.rbq_index_params_default(ctypes.byref(ip))
    assert (ip.n_lists, ip.seed, ip.kmeans_n_iters, ip.max_train_points_per_cluster) == (1024, 7, 20, 256)
    assert (ip.shard_count, ip.shard_policy, ip.kmeans_kind) == (1, 0, 0)  # round robin, balanced k-means
    sp = _lib.SearchParams()
    L.rbq_search_params_default(ctypes.byref(sp))
    assert (sp.n_probes, sp.k, sp.rerank, sp.prune, sp.seeded, sp.query_bits, sp.graph) == (20, 10, 0, 1, -1, 4, 0)


def test_scan_tile_is_one_constant():
    """The scan tile decides when the prune threshold tightens and how large candidate buffers
    are; the library, the oracle and the sharded planner must use the same value."""
    from neurosamble_b200 import _lib, sharded
    from oracle import oracle as O
    t = _lib.lib().rbq_scan_tile()
    assert t == O.SCAN_TILE == sharded.SCAN_TILE == 1024
