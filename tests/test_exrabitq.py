"""ExRaBitQ extra bits (bits_per_dim > 1): codes, factors, the extra-bit distance and searches.

The reference quantises the normalised residual to ex = bits_per_dim - 1 extra bits per
dimension (exrabitq_fused_kernel_batch, quantizer_gpu.cu:347-468) and ranks the vectors its
1-bit estimate admits by the extra-bit distance (the WithEx branch,
searcher_gpu_quantize_query.cu:405-473).  CPU tests pin the oracle by a hand-computed case and
an independent numpy restatement; GPU tests compare the library with the oracle bit for bit."""
import ctypes

import numpy as np
import pytest

from conftest import mixture

f32 = np.float32


def u32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ------------------------------------------------------------------------------------------
# independent restatements (numpy float32 scalars, python-float double sums)
# ------------------------------------------------------------------------------------------
def ex_quantize_py(y, c, ex, t):
    y, c = np.asarray(y, f32), np.asarray(c, f32)
    dp = y.size
    r = (y - c).astype(f32)
    l2 = 0.0
    for v in r:
        l2 += float(v) * float(v)
    l2 = f32(l2)
    norm = np.sqrt(l2, dtype=f32)
    mask = (1 << ex) - 1
    shift = f32(f32(1 << ex) - f32(0.5))
    planes = np.zeros((ex, dp // 32), np.uint32)
    ipn = ipr = ipc = 0.0
    for j in range(dp):
        rj = r[j]
        bit = 1 if (norm > 0 and rj > 0) else 0
        xn = f32(rj / norm) if norm > 0 else f32(0.0)
        a = abs(xn)
        e = min(int(f32(f32(f32(t) * a) + f32(1e-5))), mask)
        ipn += float(f32(f32(f32(e) + f32(0.5)) * a))
        x = e if bit else mask - e
        for p in range(ex):
            if (x >> p) & 1:
                planes[p, j >> 5] |= np.uint32(1 << (31 - (j & 31)))
        xu = f32(f32((bit << ex) | x) - shift)
        ipr += float(rj) * float(xu)
        ipc += float(c[j]) * float(xu)
    ip_resi, ip_cent, ip_norm = f32(ipr), f32(ipc), f32(ipn)
    denom = f32(np.inf) if ip_resi == 0 else ip_resi
    l2n = np.sqrt(max(l2, f32(0)), dtype=f32)
    with np.errstate(divide="ignore", invalid="ignore"):
        fadd = f32(l2 + f32(f32(f32(2.0) * l2) * ip_cent) / denom)
        inv = f32(f32(1.0) / ip_norm)
    if not np.isfinite(inv):
        inv = f32(1.0)
    fres = f32(f32(f32(-2.0) * l2n) * inv)
    return planes, np.array([fadd, fres], f32)


def byte_sum_py(q, word_row, j):
    byte = (int(word_row[j >> 2]) >> (24 - 8 * (j & 3))) & 0xFF
    s = f32(0.0)
    for jj in range(8):
        if (byte >> (7 - jj)) & 1:
            s = f32(s + q[8 * j + jj])
    return s


def ex_ip_py(q, planes):
    """Lane l: bytes j = l, l+32, ...; per byte planes p = ex-1..0 add 2^p * byte sum; butterfly."""
    q = np.asarray(q, f32)
    ex, w = planes.shape
    nb = 4 * w
    v = [f32(0.0)] * 32
    for lane in range(32):
        s = f32(0.0)
        for j in range(lane, nb, 32):
            for p in range(ex - 1, -1, -1):
                s = f32(s + f32(f32(1 << p) * byte_sum_py(q, planes[p], j)))
        v[lane] = s
    for off in (16, 8, 4, 2, 1):
        v = [f32(v[l] + v[l ^ off]) for l in range(32)]
    return v[0]


# ------------------------------------------------------------------------------------------
# CPU: the oracle against a hand-computed case and the restatements
# ------------------------------------------------------------------------------------------
def test_hand_computed_codes_and_factors(oracle):
    """r = (3, -4, 0, ..., 0), c = 0, t = 8, ex = 3: xn = (0.6, -0.8); e = (int(4.8), int(6.4)) =
    (4, 6); the second dimension's code is flipped (7 - 6 = 1); every zero coordinate gets e = 0,
    flipped to 7.  xu = (12 - 7.5, 1 - 7.5, -0.5, ...) = (4.5, -6.5, -0.5, ...), so ip_resi =
    13.5 + 26 = 39.5, f_ex_add = |r|^2 = 25 and f_ex_rescale = -10 / (4.5 * 0.6 + 6.5 * 0.8)."""
    y = np.zeros(32, f32)
    y[0], y[1] = 3.0, -4.0
    c = np.zeros(32, f32)
    planes, f2 = oracle.quantize_ex_one(y, c, 3, 8.0)
    assert planes[:, 0].tolist() == [0x7FFFFFFF, 0x3FFFFFFF, 0xBFFFFFFF]
    assert f2[0] == f32(25.0)
    ipn = f32(float(f32(f32(4.5) * f32(0.6))) + float(f32(f32(6.5) * f32(0.8))))
    assert f2[1] == f32(f32(-10.0) * f32(f32(1.0) / ipn))
    assert abs(float(f2[1]) + 10.0 / 7.9) < 1e-6
    # the one-hot query q = e_0: ip = 1 (bit 0 set), ip_x = x_0 = 4, kb = -0.5 * 15, so
    # 2^3 * 1 + 4 - 7.5 = 4.5 = <q, xu> and the estimate is (25 + |q|^2) + f_ex_rescale * 4.5
    code, _ = oracle.quantize_one(y, c)
    q = np.zeros(32, f32)
    q[0] = 1.0
    assert oracle.exact_ip(q, code) == 1.0 and oracle.ex_ip(q, planes) == 4.0


@pytest.mark.parametrize("dp,ex", [(32, 1), (64, 2), (64, 3), (96, 5), (64, 7), (128, 8)])
def test_codes_and_factors_match_an_independent_restatement(oracle, dp, ex):
    rng = np.random.default_rng(dp * 10 + ex)
    t = oracle.query_scale(dp, 7, ex)
    for it in range(6):
        c = (rng.standard_normal(dp) * 0.3).astype(f32)
        y = (c + rng.standard_normal(dp) * 0.2).astype(f32)
        if it == 0:
            y = c.copy()  # zero residual: codes 2^ex - 1 everywhere, factors 0 and -0
        pl, f2 = oracle.quantize_ex_one(y, c, ex, t)
        pl2, f22 = ex_quantize_py(y, c, ex, t)
        assert np.array_equal(pl, pl2)
        assert np.array_equal(u32(f2), u32(f22))


@pytest.mark.parametrize("dp,ex", [(32, 1), (64, 3), (256, 3), (96, 8)])
def test_extra_bit_inner_product_order(oracle, dp, ex):
    rng = np.random.default_rng(ex)
    for _ in range(5):
        q = rng.standard_normal(dp).astype(f32)
        planes = rng.integers(0, 2 ** 32, (ex, dp // 32), dtype=np.uint64).astype(np.uint32)
        assert u32(np.float32(oracle.ex_ip(q, planes))) == u32(ex_ip_py(q, planes))


def test_more_bits_estimate_distances_closer(oracle):
    """The extra-bit distance tracks the true squared distance better with every extra bit."""
    rng = np.random.default_rng(5)
    dp = 128
    err = {}
    for ex in (1, 3, 8):
        t = oracle.query_scale(dp, 7, ex)
        e = []
        for _ in range(200):
            c = (rng.standard_normal(dp) * 0.3).astype(f32)
            y = (c + rng.standard_normal(dp) * 0.2).astype(f32)
            q = (c + rng.standard_normal(dp) * 0.25).astype(f32)
            code, _ = oracle.quantize_one(y, c)
            pl, f2 = oracle.quantize_ex_one(y, c, ex, t)
            g = f32(((q.astype(np.float64) - c) ** 2).sum())
            k1 = f32(-0.5 * q.astype(np.float64).sum())
            T = f32(f32(f32(1 << ex) * f32(oracle.exact_ip(q, code))) + f32(oracle.ex_ip(q, pl)))
            T = f32(T + f32(k1 * f32((2 << ex) - 1)))
            d = f32(f32(f2[0] + g) + f32(f2[1] * T))
            true = ((q.astype(np.float64) - y) ** 2).sum()
            e.append(abs(float(d) - true) / true)
        err[ex] = float(np.mean(e))
    assert err[8] < err[3] < err[1] < 0.05


def test_search_recall_rises_with_bits(oracle):
    """Without a rerank the top-k comes from the estimator: recall@10 rises with the code bits."""
    X, Q = mixture(12000, 64, 24, 0.3, 150, seed=3)
    C, lab = oracle.kmeans(X[::3], 32, iters=4)
    lab = oracle.assign(X, C)
    P, t4 = oracle.make_rotation(64, 7), oracle.query_scale(64, 7)
    _, gt = oracle.knn_exact(X, Q, 10)
    rec = {}
    for b in (1, 3, 5, 9):
        ix = oracle.build(X, C, lab, P, t4, bits_per_dim=b, tex=oracle.ex_scale(64, 7, b - 1, t4) if b > 1 else None)
        _, i = oracle.search(ix, Q, 10, 12, 0)
        rec[b] = oracle.recall(i, gt)
    assert rec[1] + 0.2 < rec[3] < rec[5] < rec[9] and rec[9] > 0.95


def test_bits_per_dim_is_checked():
    """Argument checks run before any device work (no GPU needed)."""
    from neurosamble_b200 import _lib
    for b in (0, 10):
        p = _lib.IndexParams()
        _lib.lib().rbq_index_params_default(ctypes.byref(p))
        assert p.bits_per_dim == 1
        p.dim, p.n_lists, p.bits_per_dim = 64, 8, b
        h = ctypes.c_void_p()
        assert _lib.lib().rbq_index_create(ctypes.byref(p), ctypes.byref(h)) == 1 and not h.value
        assert b"bits_per_dim" in _lib.lib().rbq_last_error()


# ------------------------------------------------------------------------------------------
# GPU: the library against the oracle
# ------------------------------------------------------------------------------------------
def _ex_index(oracle, X, C, lab, bits, seed=7):
    from neurosamble_b200 import IndexIVFRaBitQ
    idx = IndexIVFRaBitQ(X.shape[1], C.shape[0], seed=seed, bits_per_dim=bits)
    idx.set_centroids(C)
    idx.add(X, labels=lab)
    inf = idx.info()
    oix = oracle.build(X, C, lab, idx.rotation(), idx.query_scale, bits_per_dim=bits, tex=inf.ex_scale)
    oix.t8 = oracle.query_scale(oix.dp, seed, 7)
    return idx, oix


@pytest.fixture(scope="module")
def ex_case(oracle):
    X, Q = mixture(16000, 128, 40, 0.3, 200, seed=11)
    C, _ = oracle.kmeans(X[::4], 48, iters=4)
    lab = oracle.assign(X, C)
    idx, oix = _ex_index(oracle, X, C, lab, 4)
    return idx, oix, X, Q, C, lab


@pytest.mark.gpu
@pytest.mark.parametrize("d,bits", [(128, 2), (128, 4), (100, 9), (256, 8), (32, 3)])
def test_gpu_extra_bits_and_factors_bit_exact(oracle, d, bits):
    X, _ = mixture(6000, d, 20, 0.3, 1, seed=d + bits)
    C, _ = oracle.kmeans(X[::3], 24, iters=3)
    lab = oracle.assign(X, C)
    idx, oix = _ex_index(oracle, X, C, lab, bits)
    inf = idx.info()
    assert inf.bits_per_dim == bits
    assert np.float32(inf.ex_scale) == np.float32(oracle.ex_scale(oix.dp, 7, bits - 1, idx.query_scale))
    ex = idx.export_lists()
    assert ex["ex_bits"] == bits - 1
    assert np.array_equal(ex["ids"], oix.ids) and np.array_equal(ex["codes"], oix.codes)
    assert np.array_equal(ex["ex_codes"], oix.ex_codes)
    assert np.array_equal(u32(ex["fexadd"]), u32(oix.fexadd)) and np.array_equal(u32(ex["fexr"]), u32(oix.fexr))


@pytest.mark.gpu
@pytest.mark.parametrize("mode,prune,slices,R", [(4, 1, 1, 40), (4, 0, 1, 40), (4, 1, 4, 100), (8, 1, 1, 40),
                                                 (16, 1, 1, 40), (32, 1, 3, 100), (16, 0, 1, 10)])
def test_gpu_extra_bit_scan_bit_exact(oracle, ex_case, mode, prune, slices, R):
    """Admission by the 1-bit estimate's bound (popcount or table), ranking by the extra-bit
    distance: candidates, distances and counters equal the oracle's."""
    import torch
    from neurosamble_b200 import _lib
    from neurosamble_b200.index import _ptr, _stream_ptr
    idx, oix, X, Q, C, lab = ex_case
    Qr = oracle.rotate(Q, oix.P)
    nq, nprobe = Qr.shape[0], 8
    pb = 8 if mode == 8 else 4
    qr = torch.from_numpy(Qr).cuda()
    planes = torch.empty((nq, pb, oix.dp // 32), dtype=torch.int32, device="cuda")
    delta = torch.empty(nq, dtype=torch.float32, device="cuda")
    k1 = torch.empty(nq, dtype=torch.float32, device="cuda")
    st = _stream_ptr(idx.device)
    _lib.call("rbq_query_prep", idx.handle, _ptr(qr), nq, _ptr(planes), _ptr(delta), _ptr(k1), mode, st)
    probes = torch.empty((nq, nprobe), dtype=torch.int32, device="cuda")
    g = torch.empty((nq, nprobe), dtype=torch.float32, device="cuda")
    _lib.call("rbq_coarse", idx.handle, _ptr(qr), nq, nprobe, 0, _ptr(probes), _ptr(g), st)
    ids = torch.empty((nq, R), dtype=torch.int64, device="cuda")
    dist = torch.empty((nq, R), dtype=torch.float32, device="cuda")
    stats = torch.zeros(2, dtype=torch.int64, device="cuda")
    _lib.call("rbq_scan", idx.handle, _ptr(qr), _ptr(planes), _ptr(delta), _ptr(k1), nq, _ptr(probes), _ptr(g),
              nprobe, 0, None, None, None, R, prune, slices, 0, _ptr(ids), _ptr(dist), _ptr(stats), mode, st)
    torch.cuda.synchronize()
    p2, g2 = oracle.coarse(Qr, oix.c_rot, nprobe)
    pl2, d2, k2, _ = oracle.query_prep(Qr, oix.t8 if mode == 8 else oix.t4, pb)
    oi, od, ost = oracle.scan(oix, Qr, pl2, d2, k2, p2, g2, R, prune=prune, slices=slices, with_stats=True,
                              mode=mode)
    assert np.array_equal(ids.cpu().numpy(), oi)
    assert np.array_equal(u32(dist.cpu().numpy()), u32(od))
    assert stats.cpu().tolist() == ost.tolist()


@pytest.mark.gpu
@pytest.mark.parametrize("mode,R,seeded", [(4, 0, -1), (4, 40, -1), (4, 40, 1), (8, 0, 0), (16, 0, -1), (32, 40, -1)])
def test_gpu_extra_bit_search_end_to_end(oracle, ex_case, mode, R, seeded):
    idx, oix, X, Q, C, lab = ex_case
    idx.nprobe, idx.k_rerank, idx.prune, idx.seeded, idx.query_bits = 8, R, True, seeded, mode
    try:
        for qs in (Q, Q[:3]):
            d, i = idx.search(qs, 10)
            sl = max(1, min(512 // len(qs), 8)) if len(qs) < 512 else 1
            d2, i2 = oracle.search(oix, qs, 10, 8, R, slices=sl, seeded=seeded, query_bits=mode)
            assert np.array_equal(i, i2) and np.array_equal(u32(d), u32(d2))
    finally:
        idx.query_bits, idx.seeded = 4, -1


@pytest.mark.gpu
def test_gpu_extra_bits_raise_recall_without_rerank(oracle, ex_case):
    from neurosamble_b200 import IndexIVFRaBitQ
    idx, oix, X, Q, C, lab = ex_case
    one = IndexIVFRaBitQ(X.shape[1], C.shape[0], seed=7)
    one.set_centroids(C)
    one.add(X, labels=lab)
    _, gt = oracle.knn_exact(X, Q, 10)
    rec = []
    for ix in (one, idx):
        ix.nprobe, ix.k_rerank = 12, 0
        rec.append(oracle.recall(ix.search(Q, 10)[1], gt))
    assert rec[1] > rec[0] + 0.1


@pytest.mark.gpu
def test_gpu_extra_bits_save_load_and_reference_files(oracle, ex_case, tmp_path):
    """The library's own file and the reference's (long codes: ex bits per dimension, one
    MSB-first bit stream per vector, then {f_ex_add, f_ex_rescale}) keep the extra bits."""
    from neurosamble_b200 import read_index, read_reference_index, write_index, write_reference_index
    from test_reference_format import parse_reference
    idx, oix, X, Q, C, lab = ex_case
    idx.nprobe, idx.k_rerank = 8, 0
    want = idx.search(Q, 10)
    write_index(idx, str(tmp_path / "x.rbq"))
    back = read_index(str(tmp_path / "x.rbq"))
    assert back.bits_per_dim == 4
    back.nprobe, back.k_rerank = 8, 0
    got = back.search(Q, 10)
    assert np.array_equal(got[1], want[1]) and np.array_equal(u32(got[0]), u32(want[0]))
    write_reference_index(idx, str(tmp_path / "r.index"))
    f = parse_reference(str(tmp_path / "r.index"))
    ex = idx.export_lists()
    assert f["ex"] == 3 and f["end"] == f["size"]
    # the bit stream of every vector restated from the planes
    dp, n = oix.dp, ex["ex_codes"].shape[0]
    bits = np.unpackbits(ex["ex_codes"].view(np.uint8).reshape(n, 3, -1, 4)[:, :, :, ::-1].reshape(n, 3, dp // 8),
                         axis=-1)  # [vector, plane p, dim] = bit p of the dim's code
    stream = np.stack([bits[:, 2], bits[:, 1], bits[:, 0]], axis=-1).reshape(n, dp * 3)  # MSB first
    assert np.array_equal(f["long_codes"], np.packbits(stream, axis=-1))
    assert np.array_equal(u32(f["exf"][:, 0]), u32(ex["fexadd"])) and np.array_equal(u32(f["exf"][:, 1]), u32(ex["fexr"]))
    imp = read_reference_index(str(tmp_path / "r.index"), X=X)
    assert imp.bits_per_dim == 4
    imp.nprobe, imp.k_rerank = 8, 0
    got = imp.search(Q, 10)
    assert np.array_equal(got[1], want[1]) and np.array_equal(u32(got[0]), u32(want[0]))
