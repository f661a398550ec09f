"""ctypes wrapper of the CPU oracle (oracle/rbq_oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and the
cpu_baseline / ``--impl reference`` legs of bench.py, always as the checker or the timed CPU
baseline, never as part of the product path.  Parity with the reference implementation
itself is unpinned where the reference relies on RAFT/cuSOLVER (rotation generator, t4 rows,
k-means, select_k tie order); known-answer tests pin the formulas instead.

Every function takes and returns numpy arrays (C-contiguous, exact dtypes).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "librbq_oracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_i64, _i32, _u64, _u32 = ctypes.c_int64, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint32


def compile_lib() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
            os.path.join(_HERE, "rbq_oracle.cpp")
        ):
            compile_lib()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_gaussian.argtypes = [_u64, _u32, _u64, _i64, _f64p]
        L.orc_philox.argtypes = [_u32p, _u32p, _u32p]
        L.orc_make_rotation.argtypes = [_i32, _u64, _f32p]
        L.orc_query_scale.argtypes = [_i32, _u64, _i32]
        L.orc_query_scale.restype = ctypes.c_float
        L.orc_best_rescale.argtypes = [_f64p, _i32, _i32]
        L.orc_best_rescale.restype = ctypes.c_double
        L.orc_rotate.argtypes = [_f32p, _i64, _i32, _i32, _f32p, _f32p]
        L.orc_quantize_one.argtypes = [_f32p, _f32p, _i32, _u32p, _f32p]
        L.orc_build.argtypes = [_f32p, _i64, _i32, _i32, _f32p, _f32p, _i32, _u32p,
                                _i64p, _u32p, _u32p, _f32p, _f32p, _f32p, _f32p]
        L.orc_query_prep.argtypes = [_f32p, _i64, _i32, ctypes.c_float, _i32, _u32p, _f32p, _f32p, _i8p]
        L.orc_coarse.argtypes = [_f32p, _i64, _f32p, _i32, _i32, _i32, _i32p, _f32p]
        L.orc_popcount_ip.argtypes = [_u32p, _u32p, _i32, _i32]
        L.orc_popcount_ip.restype = ctypes.c_int32
        L.orc_estimate.argtypes = [_f32p, ctypes.c_float, ctypes.c_int32, ctypes.c_float, ctypes.c_float, _f32p]
        L.orc_exact_ip.argtypes = [_f32p, _u32p, _i32]
        L.orc_exact_ip.restype = ctypes.c_float
        L.orc_scan.argtypes = [_i64p, _u32p, _u32p, _f32p, _f32p, _f32p, _i32, _f32p, _u32p,
                               _f32p, _f32p, _i64, _i32p, _f32p, _i32, ctypes.c_void_p, ctypes.c_void_p,
                               ctypes.c_void_p, _i32, _i32, _i32, _i32, _i32, _i32, _i32, ctypes.c_void_p,
                               _i64p, _f32p, _i64p, _i32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, _i32]
        L.orc_quantize_ex_one.argtypes = [_f32p, _f32p, _i32, _i32, ctypes.c_float, _u32p, _f32p]
        L.orc_quantize_ex.argtypes = [_f32p, _i64, _i32, _f32p, _u32p, _i32, ctypes.c_float, _u32p, _f32p, _f32p]
        L.orc_ex_ip.argtypes = [_f32p, _u32p, _i32, _i32]
        L.orc_ex_ip.restype = ctypes.c_float
        L.orc_bound_seed.argtypes = [_i64p, _u32p, _f32p, _f32p, _f32p, _i32, _u32p, _f32p, _f32p, _i64, _i32p,
                                     _f32p, _i32, _i32, _i32, _i32, ctypes.c_void_p, _f32p, _i32]
        L.orc_float_to_half.argtypes = [ctypes.c_void_p, _i64, ctypes.c_void_p]
        L.orc_float_to_half.restype = None
        L.orc_half_to_float.argtypes = [ctypes.c_void_p, _i64, ctypes.c_void_p]
        L.orc_half_to_float.restype = None
        L.orc_l2_exact.argtypes = [_f32p, _f32p, _i32]
        L.orc_l2_exact.restype = ctypes.c_float
        L.orc_rerank.argtypes = [_f32p, _i32, _f32p, _i64, _i64p, _i32, _i32, _f32p, _i64p]
        L.orc_knn_exact.argtypes = [_f32p, _i64, _i32, _f32p, _i64, _i32, _f32p, _i64p]
        L.orc_assign.argtypes = [_f32p, _i64, _i32, _f32p, _i32, _u32p]
        L.orc_threads.restype = ctypes.c_int
        L.orc_set_threads.argtypes = [_i32]
        _lib = L
    return _lib


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def pad_dim(d: int) -> int:
    return (d + 31) // 32 * 32


# Scan schedule constants shared with the CUDA library: vectors per tile (256 threads x 4
# vectors) and the candidate-buffer size rule cap = max(pow2(cand_cap or 1024), pow2(R + tile)).
SCAN_TILE = 1024


def _pow2(v: int) -> int:
    p = 1
    while p < v:
        p <<= 1
    return p


def default_cap(R: int, cand_cap: int = 0, tile: int = SCAN_TILE) -> int:
    return max(_pow2(cand_cap if cand_cap and cand_cap > 0 else 1024), _pow2(R + tile))


def threads() -> int:
    return lib().orc_threads()


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def gaussian(seed: int, stream: int, start: int, n: int) -> np.ndarray:
    out = np.empty(n, np.float64)
    lib().orc_gaussian(seed, stream, start, n, out)
    return out


def philox(key, ctr) -> np.ndarray:
    out = np.empty(4, np.uint32)
    lib().orc_philox(_c(key, np.uint32), _c(ctr, np.uint32), out)
    return out


def make_rotation(dp: int, seed: int) -> np.ndarray:
    P = np.empty((dp, dp), np.float32)
    lib().orc_make_rotation(dp, seed, P)
    return P


def query_scale(dp: int, seed: int, ex_bits: int = 3) -> float:
    return float(lib().orc_query_scale(dp, seed, ex_bits))


def best_rescale(o, ex_bits: int) -> float:
    o = _c(o, np.float64)
    return float(lib().orc_best_rescale(o, o.size, ex_bits))


def rotate(X, P) -> np.ndarray:
    X = _c(X, np.float32)
    n, d = X.shape
    dp = P.shape[0]
    Y = np.empty((n, dp), np.float32)
    lib().orc_rotate(X, n, d, dp, _c(P, np.float32), Y)
    return Y


def quantize_one(y, c):
    y, c = _c(y, np.float32), _c(c, np.float32)
    dp = y.size
    code = np.empty(dp // 32, np.uint32)
    f3 = np.empty(3, np.float32)
    lib().orc_quantize_one(y, c, dp, code, f3)
    return code, f3


def quantize_ex_one(y, c, ex_bits: int, t: float):
    """ExRaBitQ extra-bit planes [ex_bits, W] and (f_ex_add, f_ex_rescale) of one rotated vector."""
    y, c = _c(y, np.float32), _c(c, np.float32)
    dp = y.size
    planes = np.empty((ex_bits, dp // 32), np.uint32)
    f2 = np.empty(2, np.float32)
    lib().orc_quantize_ex_one(y, c, dp, ex_bits, np.float32(t), planes, f2)
    return planes, f2


def quantize_ex(Y, c_rot, labels, ex_bits: int, t: float):
    """Extra-bit planes [n, ex_bits, W], f_ex_add [n], f_ex_rescale [n] of rotated rows Y."""
    Y = _c(Y, np.float32)
    n, dp = Y.shape
    planes = np.empty((n, ex_bits, dp // 32), np.uint32)
    fa = np.empty(n, np.float32)
    fr = np.empty(n, np.float32)
    if n:
        lib().orc_quantize_ex(Y, n, dp, _c(c_rot, np.float32), _c(labels, np.uint32), ex_bits, np.float32(t),
                              planes, fa, fr)
    return planes, fa, fr


def ex_ip(q, planes) -> float:
    """<extra-bit code, q> of one vector's planes [ex_bits, W] in the scan's summation order."""
    planes = _c(planes, np.uint32)
    ex, w = planes.shape
    return float(lib().orc_ex_ip(_c(q, np.float32), planes, w, ex))


def ex_scale(dp: int, seed: int, ex_bits: int, t4: float, t8=None) -> float:
    """The data scale of ex_bits extra bits: the 4-bit query scale at 3, the 8-bit one at 7
    (ivf_gpu.cu:629-644), else the best-rescale mean for ex_bits (query_scale)."""
    if ex_bits == 3:
        return float(t4)
    if ex_bits == 7:
        return float(t8) if t8 is not None else query_scale(dp, seed, 7)
    return query_scale(dp, seed, ex_bits)


class OracleIndex:
    """Index arrays in list-slot order, as the CUDA library lays them out in HBM."""

    def __init__(self, d, dp, k, list_off, ids, codes, fadd, frescale, ferr, c_rot, P, t4, X):
        self.d, self.dp, self.k = d, dp, k
        self.t8 = None  # 8-bit query scale (QUANT8), query_scale(dp, seed, 7) of the index
        self.list_off, self.ids, self.codes = list_off, ids, codes
        self.fadd, self.frescale, self.ferr = fadd, frescale, ferr
        self.c_rot, self.P, self.t4, self.X = c_rot, P, t4, X
        # ExRaBitQ (bits_per_dim = ex_bits + 1 > 1): planes [n, ex_bits, W], factors [n], slot order
        self.ex_bits, self.ex_codes, self.fexadd, self.fexr, self.tex = 0, None, None, None, None

    def set_ex(self, ex_bits, ex_codes, fexadd, fexr, tex=None):
        self.ex_bits = int(ex_bits)
        self.ex_codes = _c(ex_codes, np.uint32).reshape(-1, ex_bits, self.dp // 32)
        self.fexadd, self.fexr, self.tex = _c(fexadd, np.float32), _c(fexr, np.float32), tex
        return self


def build(X, C, labels, P, t4, bits_per_dim=1, tex=None) -> OracleIndex:
    """Index of X with the given centroids and labels; bits_per_dim > 1 adds ExRaBitQ extra bits
    with data scale tex (default t4, the 4-bit query scale, which the reference uses at 4 bits)."""
    X = _c(X, np.float32)
    C = _c(C, np.float32)
    n, d = X.shape
    k = C.shape[0]
    dp = P.shape[0]
    w = dp // 32
    list_off = np.empty(k + 1, np.int64)
    ids = np.empty(n, np.uint32)
    codes = np.empty((n, w), np.uint32)
    fadd = np.empty(n, np.float32)
    fres = np.empty(n, np.float32)
    ferr = np.empty(n, np.float32)
    c_rot = np.empty((k, dp), np.float32)
    labels = _c(labels, np.uint32)
    lib().orc_build(X, n, d, dp, _c(P, np.float32), C, k, labels, list_off, ids,
                    codes, fadd, fres, ferr, c_rot)
    ix = OracleIndex(d, dp, k, list_off, ids, codes, fadd, fres, ferr, c_rot, P, t4, X)
    if bits_per_dim > 1:
        ex = bits_per_dim - 1
        t = float(t4) if tex is None else float(tex)
        Y = rotate(X[ids.astype(np.int64)], P)
        planes, fa, fr = quantize_ex(Y, c_rot, labels[ids.astype(np.int64)], ex, t)
        ix.set_ex(ex, planes, fa, fr, t)
    return ix


def query_prep(Qr, t4: float, bits: int = 4):
    """Planes [nq, bits, W], delta, k1 and int8 codes of bits-bit query codes (4: QUANT4 with t4,
    8: QUANT8 with t8)."""
    assert bits in (4, 8)
    Qr = _c(Qr, np.float32)
    nq, dp = Qr.shape
    w = dp // 32
    planes = np.empty((nq, bits, w), np.uint32)
    delta = np.empty(nq, np.float32)
    k1 = np.empty(nq, np.float32)
    codes = np.empty((nq, dp), np.int8)
    lib().orc_query_prep(Qr, nq, dp, np.float32(t4), bits, planes, delta, k1, codes)
    return planes, delta, k1, codes


def _bits_of(planes, nq, w) -> int:
    """Query code width of planes [nq, bits, w] (or the same words flattened)."""
    planes = np.asarray(planes)
    if planes.ndim == 3:
        return int(planes.shape[1])
    return 4 if nq == 0 else int(planes.size // (nq * w))


def coarse(Qr, Cr, nprobe: int):
    Qr, Cr = _c(Qr, np.float32), _c(Cr, np.float32)
    nq, dp = Qr.shape
    probes = np.empty((nq, nprobe), np.int32)
    g = np.empty((nq, nprobe), np.float32)
    lib().orc_coarse(Qr, nq, Cr, Cr.shape[0], dp, nprobe, probes, g)
    return probes, g


def popcount_ip(planes, code) -> int:
    """planes: one query's [bits, W] planes (bits = planes.size / W)."""
    code = _c(code, np.uint32)
    planes = _c(planes, np.uint32)
    return int(lib().orc_popcount_ip(planes, code, code.size, planes.size // code.size))


def estimate(f3, g, acc, delta, k1):
    out = np.empty(2, np.float32)
    lib().orc_estimate(_c(f3, np.float32), np.float32(g), int(acc), np.float32(delta), np.float32(k1), out)
    return out[0], out[1]


def exact_ip(q, code) -> float:
    code = _c(code, np.uint32)
    return float(lib().orc_exact_ip(_c(q, np.float32), code, code.size))


LUT_MODES = (16, 32)  # query_bits values of the LUT16 / LUT32 search modes


def scan(ix: OracleIndex, Qr, planes, delta, k1, probes, g, R, tile=SCAN_TILE, cap=None, prune=1,
         slices=1, shard_rank=0, shard_count=1, with_stats=False, tau0=None, init=None, owner=None, mode=None):
    """rbq_scan: top-R (ids, estimated distances) per query.  tau0 [nq] seeds every slice's
    threshold; init = (ids, dist) [nq, R] are an earlier scan's candidates slice 0 starts from;
    owner [K] (default l % shard_count) is the list -> shard map.  mode 16 / 32 (LUT16 / LUT32)
    ranks by the query-table estimate instead of the planes' popcounts (planes then hold the
    4-bit codes the query preparation made, unused); default: the planes' code width."""
    Qr = _c(Qr, np.float32)
    nq = Qr.shape[0]
    probes, g = _c(probes, np.int32), _c(g, np.float32)
    nprobe = probes.shape[1]
    if cap is None:
        cap = default_cap(R, 0, tile)
    out_ids = np.empty((nq, R), np.int64)
    out_d = np.empty((nq, R), np.float32)
    stats = np.zeros(2, np.int64)
    t0 = i0 = d0 = ow = None
    if owner is not None:
        owner = _c(owner, np.int32)
        ow = owner.ctypes.data_as(ctypes.c_void_p)
    if tau0 is not None:
        tau0 = _c(tau0, np.float32)
        t0 = tau0.ctypes.data_as(ctypes.c_void_p)
    if init is not None:
        init_i, init_d = _c(init[0], np.int64), _c(init[1], np.float32)
        assert init_i.shape == (nq, R) and init_d.shape == (nq, R)
        i0, d0 = init_i.ctypes.data_as(ctypes.c_void_p), init_d.ctypes.data_as(ctypes.c_void_p)
    if nq and nprobe:
        lib().orc_scan(ix.list_off, ix.ids, ix.codes.reshape(-1), ix.fadd, ix.frescale, ix.ferr, ix.dp, Qr,
                       _c(planes, np.uint32), _c(delta, np.float32), _c(k1, np.float32), nq, probes, g,
                       nprobe, t0, i0, d0, R, tile, cap, prune, slices, shard_rank, shard_count, ow,
                       out_ids, out_d, stats, mode if mode else _bits_of(planes, nq, ix.dp // 32), *_ex_args(ix))
    elif init is not None:
        out_ids[:], out_d[:] = merge_candidates([(init_i, init_d)], R)
    else:
        out_ids.fill(-1)
        out_d.fill(np.inf)
    if with_stats:
        return out_ids, out_d, stats
    return out_ids, out_d


def _ex_args(ix):
    """The trailing ExRaBitQ arguments of orc_scan (null pointers for a 1-bit index)."""
    ex = getattr(ix, "ex_bits", 0)
    if not ex:
        return None, None, None, 0
    return (ix.ex_codes.ctypes.data_as(ctypes.c_void_p), ix.fexadd.ctypes.data_as(ctypes.c_void_p),
            ix.fexr.ctypes.data_as(ctypes.c_void_p), ex)


def _keys(ids, d):
    """64-bit sort keys (ordered float bits << 32 | id), as the CUDA path builds them."""
    b = np.ascontiguousarray(d, np.float32).view(np.uint32).astype(np.uint64)
    ordered = np.where(b & 0x80000000, ~b & 0xFFFFFFFF, b | 0x80000000)
    k = (ordered << np.uint64(32)) | (ids.astype(np.uint64) & np.uint64(0xFFFFFFFF))
    return np.where(ids < 0, np.uint64(0xFFFFFFFFFFFFFFFF), k)


def merge_candidates(parts, R):
    """R smallest (distance, id) of several [nq, r] candidate lists (ids -1 = empty)."""
    ids = np.concatenate([p[0] for p in parts], axis=1)
    d = np.concatenate([p[1] for p in parts], axis=1)
    keys = np.sort(_keys(ids, d), axis=1)[:, :R]
    empty = keys == np.uint64(0xFFFFFFFFFFFFFFFF)
    out_i = np.where(empty, -1, (keys & np.uint64(0xFFFFFFFF)).astype(np.int64))
    ob = (keys >> np.uint64(32)).astype(np.uint32)
    bits = np.where(ob & 0x80000000, ob & 0x7FFFFFFF, ~ob).astype(np.uint32)
    out_d = np.where(empty, np.inf, bits.view(np.float32)).astype(np.float32)
    return out_i.astype(np.int64), out_d


def bound_seed(ix: OracleIndex, planes, delta, k1, probes, g, R, shard_rank=0, shard_count=1, owner=None):
    """rbq_bound_seed: per query the R-th smallest upper bound est + f_err sqrt(g) over the
    leading owned lists of `probes` holding >= R vectors (+inf if fewer)."""
    probes, g = _c(probes, np.int32), _c(g, np.float32)
    nq, nprobe = probes.shape
    out = np.empty(nq, np.float32)
    ow = None
    if owner is not None:
        owner = _c(owner, np.int32)
        ow = owner.ctypes.data_as(ctypes.c_void_p)
    if nq:
        lib().orc_bound_seed(ix.list_off, ix.codes.reshape(-1), ix.fadd, ix.frescale, ix.ferr, ix.dp,
                             _c(planes, np.uint32), _c(delta, np.float32), _c(k1, np.float32), nq, probes, g, nprobe,
                             R, shard_rank, shard_count, ow, out, _bits_of(planes, nq, ix.dp // 32))
    return out


def seeded_scan(ix: OracleIndex, Qr, planes, delta, k1, probes, g, R, tile=SCAN_TILE, cap=None, prune=1,
                slices=1, shard_rank=0, shard_count=1, with_stats=False, exchange=False, owner=None):
    """The seeded scan of rbq_search and of the sharded search: every slice starts from the
    bound seed of the query's nearest probed list (bound_seed over probes[:, :1], on the shard
    that owns that list).  exchange=False: the shard's own seed (+inf on the other shards);
    exchange=True: the minimum over the shards, i.e. the owner's seed, which the sharded
    search's all-reduce hands to every shard."""
    if not prune:
        return scan(ix, Qr, planes, delta, k1, probes, g, R, tile, cap, prune, slices, shard_rank, shard_count,
                    with_stats=with_stats, owner=owner)
    if exchange:
        tau = bound_seed(ix, planes, delta, k1, probes[:, :1], g[:, :1], R)
    else:
        tau = bound_seed(ix, planes, delta, k1, probes[:, :1], g[:, :1], R, shard_rank, shard_count, owner)
    return scan(ix, Qr, planes, delta, k1, probes, g, R, tile, cap, prune, slices, shard_rank, shard_count,
                with_stats=with_stats, tau0=tau, owner=owner)


def list_owners(policy: str, sizes, count: int) -> np.ndarray:
    """The library's list -> shard map (include/rbq.h, RBQ_SHARD_*), restated: "round_robin"
    puts list l on l % count; "balanced" takes the lists by decreasing size^2 (ties: smaller
    id) and gives each to the shard with the smallest sum of size^2 so far (ties: smaller rank)."""
    sizes = np.asarray(sizes, np.int64)
    K = sizes.size
    if count <= 1:
        return np.zeros(K, np.int32)
    if policy == "round_robin":
        return (np.arange(K) % count).astype(np.int32)
    sq = [int(s) * int(s) for s in sizes]
    order = sorted(range(K), key=lambda l: (-sq[l], l))
    load = [0] * count
    own = np.zeros(K, np.int32)
    for l in order:
        r = min(range(count), key=lambda j: (load[j], j))
        own[l] = r
        load[r] += sq[l]
    return own


def l2_exact(x, q) -> float:
    x, q = _c(x, np.float32), _c(q, np.float32)
    return float(lib().orc_l2_exact(x, q, x.size))


def rerank(X, Q, cand, k):
    X, Q = _c(X, np.float32), _c(Q, np.float32)
    cand = _c(cand, np.int64)
    nq, R = cand.shape
    out_d = np.empty((nq, k), np.float32)
    out_i = np.empty((nq, k), np.int64)
    lib().orc_rerank(X, X.shape[1], Q, nq, cand, R, k, out_d, out_i)
    return out_d, out_i


def knn_exact(X, Q, k):
    X, Q = _c(X, np.float32), _c(Q, np.float32)
    nq = Q.shape[0]
    out_d = np.empty((nq, k), np.float32)
    out_i = np.empty((nq, k), np.int64)
    lib().orc_knn_exact(X, X.shape[0], X.shape[1], Q, nq, k, out_d, out_i)
    return out_d, out_i


def assign(X, C) -> np.ndarray:
    X, C = _c(X, np.float32), _c(C, np.float32)
    labels = np.empty(X.shape[0], np.uint32)
    lib().orc_assign(X, X.shape[0], X.shape[1], C, C.shape[0], labels)
    return labels


# The list scan (rbq_search_params_t.scan_kind): batches whose probed lists are shared by at least
# this many queries on average take it under scan_kind 0 (auto).
LIST_SCAN_MIN_PAIRS_PER_LIST = 64


def uses_list_scan(scan_kind, query_bits, prune, dp, nq, nprobe, K, n_total=None, R=0) -> bool:
    """The library's choice between the tile scan and the list scan: 2 the list scan, 1 the tile
    scan, 0 (auto) the list scan for popcount modes with the prune on when nq * P >= 64 K and
    the index holds n_total >= R K vectors (R = max(rerank, k))."""
    able = query_bits in (4, 8) and bool(prune) and dp % 32 == 0 and dp <= 768
    if scan_kind == 2:
        if not able:
            raise ValueError("list scan: needs QUANT4 / QUANT8, the prune on and a padded dim <= 768")
        return True
    return (scan_kind == 0 and able and nq * nprobe >= LIST_SCAN_MIN_PAIRS_PER_LIST * K
            and (n_total is None or n_total >= R * K))


def list_scan(ix: OracleIndex, Qr, planes, delta, k1, probes, g, R, tau0, shard_rank=0, shard_count=1,
              with_stats=False, owner=None):
    """The list scan's result: every query admits a vector while its lower bound is below the
    fixed tau0[q] (no tightening), keeps the admitted vectors whose distance is <= tau0[q] and
    returns the R smallest (distance, id) keys.  One tile spanning all probed lists gives exactly
    that in scan(); a cut to R along the way cannot change the R smallest."""
    return scan(ix, Qr, planes, delta, k1, probes, g, R, tile=1 << 30, cap=(1 << 30) + (1 << 20), prune=1,
                slices=1, shard_rank=shard_rank, shard_count=shard_count, with_stats=with_stats, tau0=tau0,
                owner=owner)


def list_search_scan(ix: OracleIndex, Qr, planes, delta, k1, probes, g, R, tile=SCAN_TILE, cap=None, shard_rank=0,
                     shard_count=1, owner=None):
    """The scan of a search with scan_kind 2: (1) the bound seed over the leading probed lists
    holding >= R vectors; (2) the tile scan of the nearest probe from that seed; (3) the threshold
    for the other probes = min(seed, the nearest list's R-th distance when it found R); (4) the
    list scan of probes 1..P-1 with that fixed threshold; (5) the R smallest keys of (2) and (4).
    Returns (ids, dist, stats) like scan(..., with_stats=True)."""
    probes, g = _c(probes, np.int32), _c(g, np.float32)
    seed = bound_seed(ix, planes, delta, k1, probes, g, R, shard_rank, shard_count, owner)
    ia, da, sa = scan(ix, Qr, planes, delta, k1, probes[:, :1], g[:, :1], R, tile, cap, 1, 1, shard_rank,
                      shard_count, with_stats=True, tau0=seed, owner=owner)
    if probes.shape[1] == 1:
        return ia, da, sa
    tau1 = np.where(ia[:, R - 1] >= 0, np.minimum(seed, da[:, R - 1]), seed).astype(np.float32)
    ib, db, sb = list_scan(ix, Qr, planes, delta, k1, probes[:, 1:], g[:, 1:], R, tau1, shard_rank, shard_count,
                           with_stats=True, owner=owner)
    mi, md = merge_candidates([(ia, da), (ib, db)], R)
    return mi, md, sa + sb


def sharded_list_search_scan(ix: OracleIndex, Qr, planes, delta, k1, probes, g, R, tile=SCAN_TILE, cap=None,
                             shard_rank=0, shard_count=1, owner=None):
    """The list scan of the sharded search (neurosamble_b200.sharded) on shard `shard_rank`: the
    seed is the bound seed over the leading owned probed lists of the shard that owns the nearest
    probe; that shard scans the nearest probe by tiles from it; the threshold for the other
    probes is the minimum over the shards of min(seed, the nearest list's R-th distance); every
    shard list-scans its other owned probes with it; the shard's answer is the R smallest of
    both."""
    probes, g = _c(probes, np.int32), _c(g, np.float32)
    ranks = range(shard_count)
    own0 = (np.asarray(owner)[probes[:, 0]] if owner is not None else probes[:, 0] % shard_count)
    seed = np.min([np.where(own0 == r, bound_seed(ix, planes, delta, k1, probes, g, R, r, shard_count, owner),
                            np.float32(np.inf)) for r in ranks], axis=0).astype(np.float32)
    A = [scan(ix, Qr, planes, delta, k1, probes[:, :1], g[:, :1], R, tile, cap, 1, 1, r, shard_count,
              with_stats=True, tau0=seed, owner=owner) for r in ranks]
    ia, da, sa = A[shard_rank]
    if probes.shape[1] == 1:
        return ia, da, sa
    tau1 = np.min([np.where(a[0][:, R - 1] >= 0, np.minimum(seed, a[1][:, R - 1]), seed) for a in A],
                  axis=0).astype(np.float32)
    ib, db, sb = list_scan(ix, Qr, planes, delta, k1, probes[:, 1:], g[:, 1:], R, tau1, shard_rank, shard_count,
                           with_stats=True, owner=owner)
    mi, md = merge_candidates([(ia, da), (ib, db)], R)
    return mi, md, sa + sb


def search(ix: OracleIndex, Q, k, nprobe, rerank_depth, tile=SCAN_TILE, cap=None, prune=1, slices=1,
           shard_rank=0, shard_count=1, with_stats=False, exchange=False, seeded=-1, owner=None, query_bits=4,
           scan_kind=0):
    """Full search pipeline: rotate -> coarse -> query prep -> scan -> rerank.

    seeded (rbq_search_params_t.seeded): -1 scans in two phases (seeded_scan) when the probes
    are split into slices > 1, 0 never, 1 always; exchange=True is the sharded search's
    pipeline (two phases, threshold shared by all shards).  rerank_depth == 0 returns the
    scan's top-k estimates (the reference behaviour).  query_bits 8 (QUANT8) quantises the
    queries to 8 bits with ix.t8 (set it to query_scale(dp, seed, 7) of the index); 16 / 32
    (LUT16 / LUT32) estimate with fp16 / fp32 tables of the float query (one pass, no seed).
    scan_kind (rbq_search_params_t.scan_kind): 0 auto, 1 tile scan, 2 list scan (list_search);
    the sharded search's pipeline (exchange=True) scans by tiles."""
    Q = _c(Q, np.float32)
    Qr = rotate(Q, ix.P)
    probes, g = coarse(Qr, ix.c_rot, nprobe)
    if query_bits == 8 and getattr(ix, "t8", None) is None:
        raise ValueError("QUANT8 needs the index's 8-bit scale: set ix.t8 = query_scale(dp, seed, 7)")
    planes, delta, k1, _ = query_prep(Qr, ix.t8 if query_bits == 8 else ix.t4, 8 if query_bits == 8 else 4)
    R = rerank_depth if rerank_depth > 0 else k
    if query_bits in LUT_MODES:  # the table estimate is final: one pass, no seed
        res = scan(ix, Qr, planes, delta, k1, probes, g, R, tile, cap, prune, slices, shard_rank, shard_count,
                   with_stats=True, owner=owner, mode=query_bits)
        cand, cd = res[0], res[1]
        if rerank_depth > 0:
            dist, ids = rerank(ix.X, Q, cand, k)
        else:
            dist, ids = cd[:, :k].copy(), cand[:, :k].copy()
        return (dist, ids, res[2]) if with_stats else (dist, ids)
    two = slices > 1 if seeded < 0 else seeded > 0
    if uses_list_scan(scan_kind, query_bits, prune, ix.dp, Q.shape[0], nprobe, ix.k, int(ix.list_off[-1]), R):
        if exchange:
            res = sharded_list_search_scan(ix, Qr, planes, delta, k1, probes, g, R, tile, cap, shard_rank,
                                           shard_count, owner)
        else:
            res = list_search_scan(ix, Qr, planes, delta, k1, probes, g, R, tile, cap, shard_rank, shard_count, owner)
    elif exchange or two:
        res = seeded_scan(ix, Qr, planes, delta, k1, probes, g, R, tile, cap, prune, slices, shard_rank,
                          shard_count, with_stats=True, exchange=exchange, owner=owner)
    else:
        res = scan(ix, Qr, planes, delta, k1, probes, g, R, tile, cap, prune, slices, shard_rank,
                   shard_count, with_stats=True, owner=owner)
    cand, cd = res[0], res[1]
    if rerank_depth > 0:
        dist, ids = rerank(ix.X, Q, cand, k)
    else:
        dist, ids = cd[:, :k].copy(), cand[:, :k].copy()
    if with_stats:
        return dist, ids, res[2]
    return dist, ids


def float_to_half_bits(x) -> np.ndarray:
    """The oracle's fp32 -> fp16 rounding (round to nearest, ties to even) as uint16 bits."""
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_float_to_half(x.ctypes.data_as(ctypes.c_void_p), x.size, out.ctypes.data_as(ctypes.c_void_p))
    return out


def half_bits_to_float(h) -> np.ndarray:
    h = np.ascontiguousarray(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().orc_half_to_float(h.ctypes.data_as(ctypes.c_void_p), h.size, out.ctypes.data_as(ctypes.c_void_p))
    return out


def recall(ids, gt) -> float:
    """Mean |ids ∩ gt| / k over queries (k = gt.shape[1])."""
    k = gt.shape[1]
    hit = 0
    for a, b in zip(ids, gt):
        hit += len(set(a[:k].tolist()) & set(b.tolist()))
    return hit / float(gt.size)


def _km_update(X, lab, k, zero_empty, C):
    """M step: means of member rows, summed in ascending row order in double; empty
    clusters become zero (balanced) or keep their centre (Lloyd)."""
    sums = np.zeros((k, X.shape[1]), np.float64)
    np.add.at(sums, lab, X.astype(np.float64))
    cnt = np.bincount(lab, minlength=k).astype(np.int64)
    nz = cnt > 0
    C = C.copy()
    C[nz] = (sums[nz] / cnt[nz, None]).astype(np.float32)
    if zero_empty:
        C[~nz] = 0.0
    return C, cnt


def _km_stride(state, n):
    """Rebalancing walk stride: the next of 40 primes (smallest prime >= 61 + 64 t) not dividing n."""
    def next_prime(x):
        while True:
            if x > 1 and all(x % d for d in range(2, int(x ** 0.5) + 1)):
                return x
            x += 1
    while True:
        state[0] = (state[0] + 1) % 40
        p = next_prime(61 + 64 * state[0])
        if n % p:
            return p


def _km_adjust(X, C, lab, size, threshold, state):
    """Rebalancing pass (kmeans_balanced.cuh:443-591, adjust_centers) in ascending cluster
    order with one shared walk counter; centre math in float32, in the reference's order."""
    n, k = X.shape[0], C.shape[0]
    average = n // k
    limit = int(np.float32(average) * np.float32(threshold))
    stride = _km_stride(state, n)
    count = 0
    moved = False
    C = C.copy()
    for l in range(k):
        if size[l] > limit:
            continue
        while True:
            count += 1
            i = (stride * count) % n
            if size[lab[i]] >= average:
                break
        li = int(lab[i])
        wc = np.float32(min(int(size[l]), 7))
        v = np.float32(0.0) + wc * C[li]
        v = v + np.float32(1.0) * X[i]
        C[l] = v / (wc + np.float32(1.0))
        moved = True
    return C, moved


def _km_em(X, C, n_iters, pullback, threshold, state, lab=None, size=None, assign_fn=None):
    """EM with rebalancing (kmeans_balanced.cuh:593-704)."""
    assign_fn = assign_fn or assign
    k = C.shape[0]
    counter = pullback
    it = 0
    while it < n_iters:
        if it > 0:
            C, moved = _km_adjust(X, C, lab, size, threshold, state)
            if moved:
                if counter >= pullback:
                    counter -= pullback
                    n_iters += 1
                counter += 1
        lab = assign_fn(X, C)
        C, size = _km_update(X, lab, k, True, C)
        it += 1
    return C, lab, size


def _km_build(X, k, iters, state, assign_fn=None):
    """Labels i mod k, their means, then EM with pullback 2, threshold 0.25
    (kmeans_balanced.cuh:706-757)."""
    lab = (np.arange(X.shape[0]) % k).astype(np.uint32)
    C, size = _km_update(X, lab, k, True, np.zeros((k, X.shape[1]), np.float32))
    return _km_em(X, C, iters, 2, 0.25, state, lab, size, assign_fn)


def kmeans_balanced(X, K, iters=20, assign_fn=None):
    """Hierarchical balanced k-means (kmeans_balanced.cuh:759-1132), the deterministic
    restatement the library trains with (rbq_train, RBQ_KMEANS_BALANCED): ~sqrt(K)
    mesoclusters, fine clusters per mesocluster in proportion to its rows (at most 2n/n_meso
    rows train them), then max(iters/10, 2) fine-tuning passes.  Returns C [K, D] float32.
    assign_fn(X, C) -> uint32 labels replaces the exact E step (the bench's CPU arm passes a
    BLAS argmin for speed at 1M rows)."""
    X = _c(X, np.float32)
    n, D = X.shape
    state = [0]
    n_meso = min(K, int(np.sqrt(float(K)) + 0.5))
    _, mlab, msize = _km_build(X, n_meso, iters, state, assign_fn)
    nums = np.zeros(n_meso, np.int64)
    lists_rem, rows_rem = K, n
    nonempty_rem = int((msize > 0).sum())
    for i in range(n_meso):
        if i < n_meso - 1:
            if msize[i] == 0:
                nums[i] = 0
            else:
                nonempty_rem -= 1
                f = int(float(lists_rem * int(msize[i])) / float(rows_rem) + 0.5)
                f = min(f, lists_rem - nonempty_rem)
                nums[i] = max(f, 1)
        else:
            nums[i] = lists_rem
        lists_rem -= int(nums[i])
        rows_rem -= int(msize[i])
    csum = np.concatenate([[0], np.cumsum(nums)])
    size_max = min(int(msize.max()), (2 * n + n_meso - 1) // max(n_meso, 1))
    C = np.zeros((K, D), np.float32)
    for i in range(n_meso):
        rows = np.nonzero(mlab == i)[0][:size_max]
        if rows.size == 0:
            assert nums[i] == 0
            continue
        Ci, _, _ = _km_build(X[rows], int(nums[i]), iters, state, assign_fn)
        C[csum[i]:csum[i + 1]] = Ci
    C, _, _ = _km_em(X, C, max(iters // 10, 2), 5, 0.2, state, assign_fn=assign_fn)
    return C


def train_sample(X, K, max_train_per_list=256):
    """The evenly strided training sample rbq_train clusters: rows i * n / n_train."""
    n = X.shape[0]
    m = min(n, max_train_per_list * K)
    return _c(X, np.float32)[(np.arange(m, dtype=np.int64) * n) // m]


def kmeans(X, k, iters=10, seed=0):
    """Small deterministic Lloyd k-means for CPU-only tests (not the product's trainer)."""
    X = _c(X, np.float32)
    n = X.shape[0]
    pick = (np.arange(k, dtype=np.int64) * n) // k
    C = X[pick].copy()
    for _ in range(iters):
        lab = assign(X, C)
        sums = np.zeros((k, X.shape[1]), np.float64)
        np.add.at(sums, lab, X.astype(np.float64))
        cnt = np.bincount(lab, minlength=k)
        nz = cnt > 0
        C[nz] = (sums[nz] / cnt[nz, None]).astype(np.float32)
    return C, assign(X, C)
