"""The reference's index file (IVFGPU::save / load_transposed): layout, import and export.

The layout restated here in numpy follows gpu_index/ivf_gpu.cu:367-461 (save) and
rotator_gpu.cu:93-112 / initializer_gpu.cu:54-64; no file written by the reference itself is
available, so the byte layout is pinned by this restatement only."""
import ctypes
import struct

import numpy as np
import pytest

from conftest import mixture


def parse_reference(path):
    b = open(path, "rb").read()
    n, D, K, ex = struct.unpack_from("<4Q", b, 0)
    o = 32
    flag = b[o]
    o += 1
    t4, t8 = struct.unpack_from("<2f", b, o)
    o += 8
    sizes = np.frombuffer(b, np.uint64, K, o)
    o += 8 * K
    kind = b[o]
    o += 1
    Dp = (D + 31) // 32 * 32
    W = Dp // 32
    take = lambda dt, cnt: (np.frombuffer(b, dt, cnt, o), o + cnt * np.dtype(dt).itemsize)
    P, o = take(np.float32, Dp * Dp)
    C, o = take(np.float32, K * Dp)
    codes, o = take(np.uint32, n * W)
    fac, o = take(np.float32, n * 3)
    lc, o = take(np.uint8, n * Dp * ex // 8)
    exf, o = take(np.float32, n * 2)
    ids, o = take(np.uint32, n)
    return dict(n=n, D=D, K=K, ex=ex, flag=flag, t4=t4, t8=t8, sizes=sizes, kind=kind, P=P.reshape(Dp, Dp),
                C=C.reshape(K, Dp), codes=codes.reshape(n, W), fac=fac.reshape(n, 3), ids=ids, end=o, size=len(b),
                long_codes=lc.reshape(n, Dp * ex // 8), exf=exf.reshape(n, 2))


def _header(n, D, K, ex, kind=0):
    return struct.pack("<4Q", n, D, K, ex) + b"\x01" + struct.pack("<2f", 1.0, 2.0) + struct.pack(f"<{K}Q", *([n // K] * K)) \
        + bytes([kind])


@pytest.mark.parametrize("blob,msg", [
    (b"\x00" * 12, b"truncated"),
    (_header(8, 32, 2, 9), b"extra bits"),
    (_header(8, 32, 2, 3), b"truncated"),
    (_header(8, 32, 2, 0, kind=1), b"FHT-Kac"),
    (_header(8, 32, 2, 0) + b"\x00" * 100, b"truncated"),
    (struct.pack("<4Q", 8, 0, 2, 0) + b"\x00" * 64, b"bad header"),
])
def test_import_rejects_malformed_files(tmp_path, blob, msg):
    """Host-side checks, before any device work (runs without a GPU)."""
    from neurosamble_b200 import _lib
    p = tmp_path / "r.index"
    p.write_bytes(blob)
    h = ctypes.c_void_p()
    st = _lib.lib().rbq_import_reference(str(p).encode(), 0, None, 0, 0, 1, 0, ctypes.byref(h))
    assert st == 6 and not h.value
    assert msg in _lib.lib().rbq_last_error()


@pytest.mark.gpu
def test_export_layout_and_import_round_trip(oracle, tmp_path):
    from neurosamble_b200 import IndexIVFRaBitQ, read_reference_index, write_reference_index
    X, Q = mixture(12000, 100, 30, 0.3, 150, seed=17)
    C, _ = oracle.kmeans(X[::4], 48, iters=4)
    lab = oracle.assign(X, C)
    idx = IndexIVFRaBitQ(100, 48, seed=7)
    idx.set_centroids(C)
    idx.add(X, labels=lab)
    path = tmp_path / "ref.index"
    write_reference_index(idx, str(path))
    f = parse_reference(str(path))
    ex = idx.export_lists()
    Cg, Cr = idx.centroids()
    assert (f["n"], f["D"], f["K"], f["ex"], f["flag"], f["kind"]) == (12000, 100, 48, 0, 1, 0)
    assert f["end"] == f["size"]
    assert np.float32(f["t4"]) == np.float32(idx.query_scale)
    assert np.array_equal(f["sizes"], np.diff(ex["list_off"]).astype(np.uint64))
    assert np.array_equal(f["P"], idx.rotation()) and np.array_equal(f["C"], Cr)
    assert np.array_equal(f["codes"], ex["codes"]) and np.array_equal(f["ids"], ex["ids"])
    assert np.array_equal(f["fac"], np.stack([ex["fadd"], ex["frescale"], ex["ferr"]], 1))
    # import with the raw vectors: the same search, rerank included
    back = read_reference_index(str(path), X=X)
    for a in (idx, back):
        a.nprobe, a.k_rerank = 10, 40
    d0, i0 = idx.search(Q, 10)
    d1, i1 = back.search(Q, 10)
    assert np.array_equal(i0, i1) and np.array_equal(d0.view(np.uint32), d1.view(np.uint32))
    # without them: estimator-order search only
    bare = read_reference_index(str(path))
    idx.k_rerank = bare.k_rerank = 0
    bare.nprobe = 10
    d0, i0 = idx.search(Q, 10)
    d2, i2 = bare.search(Q, 10)
    assert np.array_equal(i0, i2) and np.array_equal(d0.view(np.uint32), d2.view(np.uint32))
    bare.k_rerank = 40
    with pytest.raises(RuntimeError, match="raw vectors"):
        bare.search(Q, 10)
    # as two balanced shards: each holds its lists and searches them like the oracle
    oix = oracle.build(X, C, lab, idx.rotation(), idx.query_scale)
    want = oracle.list_owners("balanced", f["sizes"].astype(np.int64), 2)
    for r in range(2):
        sh = read_reference_index(str(path), X=X, shard_rank=r, shard_count=2, shard_policy="balanced")
        assert np.array_equal(sh.list_owners(), want)
        sh.nprobe, sh.k_rerank = 10, 40
        d, i = sh.search(Q, 10)
        d2, i2 = oracle.search(oix, Q, 10, 10, 40, shard_rank=r, shard_count=2, owner=want)
        assert np.array_equal(i, i2) and np.array_equal(d.view(np.uint32), d2.view(np.uint32))
