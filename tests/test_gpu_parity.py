"""GPU parity: every stage of librbq.so (called through the C ABI) against the CPU oracle on
the same seeded inputs.  Integer and index outputs must be bit-exact; float outputs are
compared bit for bit as well, because both sides evaluate the same operation order (the
tolerance the path allows, 1e-4 relative on distances, is asserted in addition)."""
import ctypes

import numpy as np
import pytest

from conftest import mixture

pytestmark = pytest.mark.gpu

REL_TOL = 1e-4  # distance tolerance of the north star


def _torch():
    import torch
    return torch


def dev(a):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def stream():
    torch = _torch()
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


def call(name, *args):
    from neurosamble_b200 import _lib
    _lib.call(name, *args)
    _torch().cuda.synchronize()


def make_index(oracle, X, C, lab, seed=7):
    from neurosamble_b200 import IndexIVFRaBitQ
    idx = IndexIVFRaBitQ(X.shape[1], C.shape[0], seed=seed)
    idx.set_centroids(C)
    idx.add(X, labels=lab)
    oix = oracle.build(X, C, lab, idx.rotation(), idx.query_scale)
    return idx, oix


@pytest.fixture(scope="module")
def case(oracle):
    X, Q = mixture(20000, 128, 48, 0.3, 300, seed=1)
    C, _ = oracle.kmeans(X[::4], 64, iters=4)
    lab = oracle.assign(X, C)
    idx, oix = make_index(oracle, X, C, lab)
    return idx, oix, X, Q, C, lab


def test_constants_match_oracle(oracle, case):
    idx, oix, X, Q, C, lab = case
    assert np.array_equal(u32(idx.rotation()), u32(oracle.make_rotation(128, 7)))
    assert np.float32(idx.query_scale).view(np.uint32) == np.float32(oracle.query_scale(128, 7)).view(np.uint32)
    Cg, Crg = idx.centroids()
    assert np.array_equal(u32(Crg), u32(oix.c_rot))


def test_rotation_outputs_bit_exact(oracle, case):
    idx, oix, X, Q, C, lab = case
    torch = _torch()
    for rows in (Q, X[:1000], X[:1]):
        x = dev(rows)
        y = torch.empty((rows.shape[0], 128), dtype=torch.float32, device="cuda")
        call("rbq_rotate", idx.handle, ptr(x), rows.shape[0], ptr(y), stream())
        assert np.array_equal(u32(y.cpu().numpy()), u32(oracle.rotate(rows, oix.P)))


def test_build_layout_codes_factors_bit_exact(case):
    idx, oix, X, Q, C, lab = case
    ex = idx.export_lists()
    assert np.array_equal(ex["list_off"], oix.list_off)
    assert np.array_equal(ex["ids"], oix.ids)
    assert np.array_equal(ex["codes"], oix.codes)
    for k in ("fadd", "frescale", "ferr"):
        assert np.array_equal(u32(ex[k]), u32(getattr(oix, k))), k


def test_gpu_assignment_matches_oracle(oracle, case):
    from neurosamble_b200 import IndexIVFRaBitQ
    idx, oix, X, Q, C, lab = case
    idx2 = IndexIVFRaBitQ(128, 64, seed=7)
    idx2.set_centroids(C)
    idx2.add(X)  # labels assigned on the GPU
    ex = idx2.export_lists()
    assert np.array_equal(ex["list_off"], oix.list_off)
    assert np.array_equal(ex["ids"], oix.ids)


def _query_stage(idx, Qr_np, bits=4):
    torch = _torch()
    nq, dp = Qr_np.shape
    qr = dev(Qr_np)
    planes = torch.empty((nq, bits, dp // 32), dtype=torch.int32, device="cuda")
    delta = torch.empty(nq, dtype=torch.float32, device="cuda")
    k1 = torch.empty(nq, dtype=torch.float32, device="cuda")
    call("rbq_query_prep", idx.handle, ptr(qr), nq, ptr(planes), ptr(delta), ptr(k1), planes.shape[1], stream())
    return qr, planes, delta, k1


def test_query_quantisation_bit_exact(oracle, case):
    idx, oix, X, Q, C, lab = case
    Qr = oracle.rotate(Q, oix.P)
    _, planes, delta, k1 = _query_stage(idx, Qr)
    p2, d2, k2, _ = oracle.query_prep(Qr, oix.t4)
    assert np.array_equal(u32(planes.cpu().numpy()), p2)
    assert np.array_equal(u32(delta.cpu().numpy()), u32(d2))
    assert np.array_equal(u32(k1.cpu().numpy()), u32(k2))


@pytest.mark.parametrize("nprobe", [1, 8, 64])
def test_coarse_probes_bit_exact(oracle, case, nprobe):
    idx, oix, X, Q, C, lab = case
    torch = _torch()
    Qr = oracle.rotate(Q, oix.P)
    qr = dev(Qr)
    probes = torch.empty((Q.shape[0], nprobe), dtype=torch.int32, device="cuda")
    g = torch.empty((Q.shape[0], nprobe), dtype=torch.float32, device="cuda")
    call("rbq_coarse", idx.handle, ptr(qr), Q.shape[0], nprobe, 0, ptr(probes), ptr(g), stream())
    p2, g2 = oracle.coarse(Qr, oix.c_rot, nprobe)
    assert np.array_equal(probes.cpu().numpy(), p2)
    assert np.array_equal(u32(g.cpu().numpy()), u32(g2))


def test_popcount_inner_products_and_estimates_bit_exact(oracle, case):
    idx, oix, X, Q, C, lab = case
    torch = _torch()
    Qr = oracle.rotate(Q[:4], oix.P)
    _, planes, delta, k1 = _query_stage(idx, Qr)
    pl_np = u32(planes.cpu().numpy())
    dl, kk = delta.cpu().numpy(), k1.cpu().numpy()
    for q in range(4):
        for l in (0, 5, 63):
            n = int(oix.list_off[l + 1] - oix.list_off[l])
            if n == 0:
                continue
            acc = torch.empty(n, dtype=torch.int32, device="cuda")
            est = torch.empty(n, dtype=torch.float32, device="cuda")
            low = torch.empty(n, dtype=torch.float32, device="cuda")
            g = np.float32(0.37 + 0.01 * l)
            call("rbq_list_estimates", idx.handle, ptr(planes[q]), float(dl[q]), float(kk[q]), float(g), l, ptr(acc),
                 ptr(est), ptr(low), 4, stream())
            acc_np, est_np, low_np = acc.cpu().numpy(), est.cpu().numpy(), low.cpu().numpy()
            for v in range(n):
                s = int(oix.list_off[l]) + v
                a = oracle.popcount_ip(pl_np[q], oix.codes[s])
                assert acc_np[v] == a
                f3 = np.array([oix.fadd[s], oix.frescale[s], oix.ferr[s]], np.float32)
                e, lo = oracle.estimate(f3, g, a, dl[q], kk[q])
                assert u32(np.float32(e)) == u32(est_np[v]) and u32(np.float32(lo)) == u32(low_np[v])


def _scan(idx, oracle, oix, Q, nprobe, R, prune, slices, cap=0, bits=4):
    torch = _torch()
    nq = Q.shape[0]
    Qr = oracle.rotate(Q, oix.P)
    qr, planes, delta, k1 = _query_stage(idx, Qr, bits)
    probes = torch.empty((nq, nprobe), dtype=torch.int32, device="cuda")
    g = torch.empty((nq, nprobe), dtype=torch.float32, device="cuda")
    call("rbq_coarse", idx.handle, ptr(qr), nq, nprobe, 0, ptr(probes), ptr(g), stream())
    ids = torch.empty((nq, R), dtype=torch.int64, device="cuda")
    dist = torch.empty((nq, R), dtype=torch.float32, device="cuda")
    stats = torch.zeros(2, dtype=torch.int64, device="cuda")
    call("rbq_scan", idx.handle, ptr(qr), ptr(planes), ptr(delta), ptr(k1), nq, ptr(probes), ptr(g), nprobe, 0, None, None, None, R,
         prune, slices, cap, ptr(ids), ptr(dist), ptr(stats), bits, stream())
    p2, g2 = oracle.coarse(Qr, oix.c_rot, nprobe)
    pl2, d2, k2, _ = oracle.query_prep(Qr, oix.t4 if bits == 4 else oracle.query_scale(oix.dp, 7, 7), bits)
    cap_o = oracle.default_cap(R, cap)
    oi, od, ost = oracle.scan(oix, Qr, pl2, d2, k2, p2, g2, R, oracle.SCAN_TILE, cap_o, prune, slices, with_stats=True)
    return ids.cpu().numpy(), dist.cpu().numpy(), stats.cpu().numpy(), oi, od, ost


@pytest.mark.parametrize("prune,slices,R,cap", [(1, 1, 10, 0), (1, 1, 40, 0), (0, 1, 40, 0), (1, 4, 40, 0),
                                                 (1, 1, 40, 512), (1, 3, 100, 2048), (0, 8, 10, 0)])
def test_scan_candidates_bit_exact(oracle, case, prune, slices, R, cap):
    idx, oix, X, Q, C, lab = case
    gi, gd, gst, oi, od, ost = _scan(idx, oracle, oix, Q, 8, R, prune, slices, cap)
    assert np.array_equal(gi, oi)
    assert np.array_equal(u32(gd), u32(od))
    assert gst.tolist() == ost.tolist()


def test_rerank_bit_exact(oracle, case):
    idx, oix, X, Q, C, lab = case
    torch = _torch()
    rng = np.random.default_rng(2)
    cand = rng.integers(0, X.shape[0], (Q.shape[0], 40)).astype(np.int64)
    cand[:, 30:] = -1
    ci, q = dev(cand), dev(Q)
    d = torch.empty((Q.shape[0], 10), dtype=torch.float32, device="cuda")
    i = torch.empty((Q.shape[0], 10), dtype=torch.int64, device="cuda")
    call("rbq_rerank", idx.handle, ptr(q), Q.shape[0], ptr(ci), 40, 10, ptr(d), ptr(i), stream())
    d2, i2 = oracle.rerank(X, Q, cand, 10)
    assert np.array_equal(i.cpu().numpy(), i2)
    assert np.array_equal(u32(d.cpu().numpy()), u32(d2))


@pytest.mark.parametrize("nprobe,R,prune", [(8, 40, 1), (8, 0, 1), (64, 40, 0), (3, 100, 1)])
def test_search_end_to_end(oracle, case, nprobe, R, prune):
    idx, oix, X, Q, C, lab = case
    idx.nprobe, idx.k_rerank, idx.prune = nprobe, R, bool(prune)
    d, i = idx.search(Q, 10)
    d2, i2 = oracle.search(oix, Q, 10, nprobe, R, prune=prune)
    assert np.array_equal(i, i2)
    assert np.array_equal(u32(d), u32(d2))
    fin = np.isfinite(d2)
    assert np.allclose(d[fin], d2[fin], rtol=REL_TOL, atol=0)
    _, gt = oracle.knn_exact(X, Q, 10)
    assert oracle.recall(i, gt) == oracle.recall(i2, gt)


@pytest.mark.parametrize("nq", [1, 2, 33, 64])
def test_small_batches_use_probe_slices(oracle, case, nq):
    idx, oix, X, Q, C, lab = case
    idx.nprobe, idx.k_rerank, idx.prune = 16, 40, True
    d, i = idx.search(Q[:nq], 10)
    sl = max(1, min(512 // nq, 16))
    d2, i2 = oracle.search(oix, Q[:nq], 10, 16, 40, prune=1, slices=sl)
    assert np.array_equal(i, i2)
    assert np.array_equal(u32(d), u32(d2))


def test_search_host_matches_device_search(case):
    idx, oix, X, Q, C, lab = case
    idx.nprobe, idx.k_rerank = 8, 40
    d, i = idx.search(Q, 10)
    dh, ih = idx.search_host(Q, 10)
    assert np.array_equal(i, ih) and np.array_equal(u32(d), u32(dh))


def test_search_host_in_overlapped_chunks(case):
    """Batches of >= 4096 host queries run in chunks whose copies overlap the search; the
    results equal one device-side search of the whole batch."""
    idx, oix, X, Q, C, lab = case
    Qb = np.ascontiguousarray(np.tile(Q, (30, 1))[:8999])
    Qb[300:] += np.float32(1e-3) * np.random.default_rng(3).standard_normal(Qb[300:].shape).astype(np.float32)
    idx.nprobe, idx.k_rerank = 8, 40
    d, i = idx.search(Qb, 10)
    dh, ih = idx.search_host(Qb, 10)
    assert np.array_equal(i, ih) and np.array_equal(u32(d), u32(dh))


def test_torch_inputs_stay_on_device(case):
    torch = _torch()
    idx, oix, X, Q, C, lab = case
    idx.nprobe, idx.k_rerank = 8, 40
    d, i = idx.search(torch.from_numpy(Q).cuda(), 10)
    assert d.is_cuda and i.is_cuda and i.dtype == torch.int64
    d2, i2 = idx.search(Q, 10)
    assert np.array_equal(i.cpu().numpy(), i2)


def test_save_load_round_trip(tmp_path, case):
    from neurosamble_b200 import read_index, write_index
    idx, oix, X, Q, C, lab = case
    idx.nprobe, idx.k_rerank = 8, 40
    d, i = idx.search(Q, 10)
    path = tmp_path / "a.rbq"
    write_index(idx, str(path))
    idx2 = read_index(str(path))
    idx2.nprobe, idx2.k_rerank = 8, 40
    d2, i2 = idx2.search(Q, 10)
    assert np.array_equal(i, i2) and np.array_equal(u32(d), u32(d2))
    assert idx2.ntotal == X.shape[0]


def test_incremental_add_matches_single_add(oracle, case):
    from neurosamble_b200 import IndexIVFRaBitQ
    idx, oix, X, Q, C, lab = case
    idx2 = IndexIVFRaBitQ(128, 64, seed=7)
    idx2.set_centroids(C)
    idx2.add(X[:7000], labels=lab[:7000])
    idx2.add(X[7000:], labels=lab[7000:])
    ex, ex2 = idx.export_lists(), idx2.export_lists()
    for k in ex:
        assert np.array_equal(ex[k], ex2[k]), k


def test_errors_raise_runtime_error(case):
    idx, oix, X, Q, C, lab = case
    idx.nprobe = 65
    with pytest.raises(RuntimeError, match="n_probes"):
        idx.search(Q[:2], 10)
    idx.nprobe = 8
    with pytest.raises(RuntimeError):
        idx.search(np.zeros((2, 7), np.float32), 10)


@pytest.mark.parametrize("d,n,k", [(100, 3000, 16), (768, 2000, 8), (32, 500, 4)])
def test_other_dimensions(oracle, d, n, k):
    X, Q = mixture(n, d, 6, 0.3, 40, seed=d)
    C, _ = oracle.kmeans(X, k, iters=3)
    lab = oracle.assign(X, C)
    idx, oix = make_index(oracle, X, C, lab, seed=5)
    ex = idx.export_lists()
    assert np.array_equal(ex["codes"], oix.codes)
    assert np.array_equal(u32(ex["ferr"]), u32(oix.ferr))
    idx.nprobe, idx.k_rerank = min(4, k), 20
    dd, ii = idx.search(Q, 5)
    d2, i2 = oracle.search(oix, Q, 5, min(4, k), 20, prune=1)
    assert np.array_equal(ii, i2) and np.array_equal(u32(dd), u32(d2))


def test_empty_lists_and_padding(oracle):
    X, Q = mixture(50, 64, 2, 0.3, 3, seed=9)
    C = np.concatenate([X[:2], X[:2] + 5.0]).astype(np.float32)
    lab = oracle.assign(X, C)
    idx, oix = make_index(oracle, X, C, lab)
    assert (np.diff(oix.list_off) == 0).any()
    idx.nprobe, idx.k_rerank, idx.prune = 4, 0, False
    d, i = idx.search(Q, 80)
    d2, i2 = oracle.search(oix, Q, 80, 4, 0, prune=0)
    assert np.array_equal(i, i2)
    assert (i == -1).any() and np.all(np.isinf(d[i == -1]))


def test_gpu_kmeans_is_deterministic():
    from neurosamble_b200 import IndexIVFRaBitQ
    X, Q = mixture(30000, 64, 40, 0.3, 10, seed=3)
    cs = []
    for _ in range(2):
        idx = IndexIVFRaBitQ(64, 32, seed=1, kmeans_iters=5)
        idx.train(X)
        cs.append(idx.centroids()[0])
    assert np.array_equal(u32(cs[0]), u32(cs[1]))


def test_config1_parity_and_recall(oracle):
    """Benchmark config 1 shape at full size: 100k x 128, K = 256, P = 16, k = 10, R = 40."""
    from neurosamble_b200 import IndexIVFRaBitQ
    X, Q = mixture(100000, 128, 256, 0.3, 1000, seed=11)
    idx = IndexIVFRaBitQ(128, 256, seed=7, kmeans_iters=10)
    idx.train(X)
    idx.add(X)
    C, _ = idx.centroids()
    lab = oracle.assign(X, C)
    oix = oracle.build(X, C, lab, idx.rotation(), idx.query_scale)
    ex = idx.export_lists()
    assert np.array_equal(ex["ids"], oix.ids) and np.array_equal(ex["codes"], oix.codes)
    idx.nprobe, idx.k_rerank = 16, 40
    d, i = idx.search(Q, 10)
    d2, i2 = oracle.search(oix, Q, 10, 16, 40, prune=1)
    assert np.array_equal(i, i2) and np.array_equal(u32(d), u32(d2))
    _, gt = oracle.knn_exact(X, Q, 10)
    assert oracle.recall(i, gt) == oracle.recall(i2, gt)


def _near_duplicates(n, d, nq, spread, seed):
    """Rows that all point almost the same way (a common unit vector plus a small spread), like
    the mean-pooled embeddings of a randomly initialised encoder: every centroid is nearly
    equidistant from every query, so tf32 rounding reorders the coarse scores."""
    rng = np.random.default_rng(seed)
    base = rng.standard_normal(d).astype(np.float32)
    X = base[None, :] + np.float32(spread) * rng.standard_normal((n, d)).astype(np.float32)
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    Q = X[rng.integers(0, n, nq)] + np.float32(spread / 4) * rng.standard_normal((nq, d)).astype(np.float32)
    Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    return np.ascontiguousarray(X), np.ascontiguousarray(Q)


@pytest.mark.parametrize("spread", [1e-2, 1e-3])
def test_near_duplicate_rows_keep_exact_probes_and_search(oracle, spread):
    """With the tf32 score error comparable to the gaps between centroid distances, the
    shortlist's error bound sends queries to the exact pass over all lists: probes, the nearest-
    centroid assignment and the whole search still equal the oracle's exact computation."""
    torch = _torch()
    from neurosamble_b200 import IndexIVFRaBitQ
    X, Q = _near_duplicates(20000, 256, 500, spread, seed=17)
    idx = IndexIVFRaBitQ(256, 128, seed=7, kmeans_iters=4)
    idx.train(X)
    idx.add(X)
    C, _ = idx.centroids()
    ex = idx.export_lists()
    lab = np.repeat(np.arange(128, dtype=np.uint32), np.diff(ex["list_off"]))[np.argsort(ex["ids"], kind="stable")]
    assert np.array_equal(lab, oracle.assign(X, C))  # GPU assignment = exact nearest centroid
    oix = oracle.build(X, C, lab, idx.rotation(), idx.query_scale)
    Qr = oracle.rotate(Q, oix.P)
    for nprobe in (8, 48):
        probes = torch.empty((len(Q), nprobe), dtype=torch.int32, device="cuda")
        g = torch.empty((len(Q), nprobe), dtype=torch.float32, device="cuda")
        call("rbq_coarse", idx.handle, ptr(dev(Qr)), len(Q), nprobe, 0, ptr(probes), ptr(g), stream())
        p2, g2 = oracle.coarse(Qr, oix.c_rot, nprobe)
        assert np.array_equal(probes.cpu().numpy(), p2)
        assert np.array_equal(u32(g.cpu().numpy()), u32(g2))
    idx.nprobe, idx.k_rerank = 48, 200
    d, i = idx.search(Q, 20)
    d2, i2 = oracle.search(oix, Q, 20, 48, 200, prune=1)
    assert np.array_equal(i, i2) and np.array_equal(u32(d), u32(d2))


@pytest.mark.parametrize("d,K,nq,nprobes", [(128, 2500, 300, (1, 30, 200)), (256, 4096, 129, (8, 64)),
                                             (96, 3000, 77, (16,))])
def test_fused_coarse_shortlist_probes_bit_exact(oracle, d, K, nq, nprobes):
    """K >= 2048 takes the fused tensor-core scores + shortlist kernel (no [nq, K] score matrix):
    probes and their exact distances equal the oracle's exact top-P, for ragged K and batches."""
    torch = _torch()
    from neurosamble_b200 import IndexIVFRaBitQ
    X, Q = mixture(K * 4, d, K, 0.2, nq, seed=23)
    idx = IndexIVFRaBitQ(d, K, seed=7)
    C = X[np.arange(K) * 4].copy()
    idx.set_centroids(C)
    P = idx.rotation()
    dp = P.shape[0]
    Cr = oracle.rotate(C, P)
    Qr = oracle.rotate(Q, P)
    for nprobe in nprobes:
        probes = torch.empty((nq, nprobe), dtype=torch.int32, device="cuda")
        g = torch.empty((nq, nprobe), dtype=torch.float32, device="cuda")
        call("rbq_coarse", idx.handle, ptr(dev(Qr)), nq, nprobe, 0, ptr(probes), ptr(g), stream())
        p2, g2 = oracle.coarse(Qr, Cr, nprobe)
        assert np.array_equal(probes.cpu().numpy(), p2), nprobe
        assert np.array_equal(u32(g.cpu().numpy()), u32(g2)), nprobe
    assert dp % 32 == 0


def _config2_data(n=1_000_000, d=256, centres=4096, sigma=0.25, nq=10_000, qsigma=0.05, seed=2024):
    """Benchmark config 2's generator (the bench's make_data): float32 mixture rows in chunks."""
    rng = np.random.default_rng(seed)
    cent = rng.standard_normal((centres, d), dtype=np.float32)
    X = np.empty((n, d), np.float32)
    for a in range(0, n, 1 << 17):
        b = min(n, a + (1 << 17))
        X[a:b] = cent[rng.integers(0, centres, b - a)]
        X[a:b] += np.float32(sigma) * rng.standard_normal((b - a, d), dtype=np.float32)
        X[a:b] /= np.linalg.norm(X[a:b], axis=1, keepdims=True)
    src = rng.integers(0, n, nq)
    Q = X[src] + np.float32(qsigma) * rng.standard_normal((nq, d), dtype=np.float32)
    Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    return X, np.ascontiguousarray(Q, np.float32)


def test_config2_parity_at_full_size(oracle):
    """The headline configuration at full size: 1M x 256, K = 1024 (balanced k-means, the
    default trainer), P = 32, k = 10, R = 200 (the depth the benchmark settles on).  The whole
    10,000-query batch is searched on the GPU, as the benchmark does; the oracle builds its own
    index from the rows, the GPU's centroids and the assignment, and searches the first 300
    queries.  Codes, factors, ids, distances and recall must agree exactly."""
    from neurosamble_b200 import IndexIVFRaBitQ
    X, Q = _config2_data()
    idx = IndexIVFRaBitQ(256, 1024, seed=7)
    idx.train(X)
    idx.add(X)
    C, _ = idx.centroids()
    ex = idx.export_lists()
    # the GPU's assignment, read back from its lists, checked on a sample of rows (the exact
    # assignment of all 1M rows on the CPU would dominate the test's time)
    lab = np.repeat(np.arange(1024, dtype=np.uint32), np.diff(ex["list_off"]))[np.argsort(ex["ids"], kind="stable")]
    rows = np.arange(0, X.shape[0], 997)
    assert np.array_equal(oracle.assign(X[rows], C), lab[rows])
    oix = oracle.build(X, C, lab, idx.rotation(), idx.query_scale)
    assert np.array_equal(ex["list_off"], oix.list_off) and np.array_equal(ex["ids"], oix.ids)
    assert np.array_equal(ex["codes"], oix.codes)
    for f in ("fadd", "frescale", "ferr"):
        assert np.array_equal(u32(ex[f]), u32(getattr(oix, f))), f
    idx.nprobe, idx.k_rerank = 32, 200
    d, i = idx.search(Q, 10)
    ns = 300
    d2, i2 = oracle.search(oix, Q[:ns], 10, 32, 200, prune=1)
    assert np.array_equal(i[:ns], i2)
    assert np.array_equal(u32(d[:ns]), u32(d2))
    fin = np.isfinite(d2)
    assert np.all(np.abs(d[:ns][fin] - d2[fin]) <= REL_TOL * np.abs(d2[fin]))
    _, gt = oracle.knn_exact(X, Q[:ns], 10)
    r_gpu, r_orc = oracle.recall(i[:ns], gt), oracle.recall(i2, gt)
    assert r_gpu == r_orc and r_gpu >= 0.95


@pytest.mark.parametrize("d,K,nq", [(256, 1024, 300), (128, 300, 129), (32, 64, 1), (768, 256, 200), (100, 40, 7)])
def test_tensor_core_scores_match_fp32(oracle, d, K, nq):
    """tcgen05 kind::tf32 scores vs the fp32 CUDA-core scores; tf32 keeps 10 mantissa bits, so
    |diff| <= 2e-3 * (|c|^2 + 2 |q| |c|) is asserted, and no device wait may time out."""
    torch = _torch()
    from neurosamble_b200 import IndexIVFRaBitQ
    X, Q = mixture(max(4 * K, 2000), d, 8, 0.3, nq, seed=K)
    C, _ = oracle.kmeans(X, K, iters=2)
    idx = IndexIVFRaBitQ(d, K, seed=3)
    idx.set_centroids(C)
    dp = idx.info().padded_dim
    qr = torch.empty((nq, dp), dtype=torch.float32, device="cuda")
    q = dev(Q)
    call("rbq_rotate", idx.handle, ptr(q), nq, ptr(qr), stream())
    s_tc = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    s_fp = torch.empty((nq, K), dtype=torch.float32, device="cuda")
    call("rbq_coarse_scores", idx.handle, ptr(qr), nq, ptr(s_tc), 1, stream())
    call("rbq_coarse_scores", idx.handle, ptr(qr), nq, ptr(s_fp), 0, stream())
    call("rbq_check_errors", idx.handle)
    a, b = s_tc.cpu().numpy(), s_fp.cpu().numpy()
    _, Cr = idx.centroids()
    bound = 2e-3 * ((Cr * Cr).sum(1)[None, :] + 2.0 * np.linalg.norm(qr.cpu().numpy(), axis=1)[:, None]
                    * np.linalg.norm(Cr, axis=1)[None, :]) + 1e-6
    assert np.all(np.isfinite(a))
    assert np.all(np.abs(a - b) <= bound), float(np.max(np.abs(a - b) - bound))


@pytest.mark.parametrize("seeded,split", [(1, 1), (1, 3), (0, 4), (-1, 2)])
def test_search_seeded_two_phase(oracle, case, seeded, split):
    """rbq_search_params_t.seeded: the nearest list scanned first, its candidates and R-th
    estimate seeding the rest (on, or auto when the probes are split), or one pass (0),
    bit-exact against the oracle."""
    idx, oix, X, Q, C, lab = case
    idx.nprobe, idx.k_rerank, idx.prune, idx.probe_split, idx.seeded = 12, 40, True, split, seeded
    try:
        d, i = idx.search(Q, 10)
    finally:
        idx.probe_split, idx.seeded = 0, -1
    d2, i2 = oracle.search(oix, Q, 10, 12, 40, prune=1, slices=split, seeded=seeded)
    assert np.array_equal(i, i2)
    assert np.array_equal(u32(d), u32(d2))


def test_scan_from_a_seeded_threshold(oracle, case):
    """rbq_scan's seeds: every slice starts from the per-query threshold tau0; slice 0 also from
    the initial candidates (an earlier scan's), which the result then includes."""
    torch = _torch()
    idx, oix, X, Q, C, lab = case
    nq, nprobe, R = Q.shape[0], 10, 30
    Qr = oracle.rotate(Q, oix.P)
    qr, planes, delta, k1 = _query_stage(idx, Qr)
    probes = torch.empty((nq, nprobe), dtype=torch.int32, device="cuda")
    g = torch.empty((nq, nprobe), dtype=torch.float32, device="cuda")
    call("rbq_coarse", idx.handle, ptr(qr), nq, nprobe, 0, ptr(probes), ptr(g), stream())
    p2, g2 = oracle.coarse(Qr, oix.c_rot, nprobe)
    pl2, d2, k2, _ = oracle.query_prep(Qr, oix.t4)
    ai, ad = oracle.scan(oix, Qr, pl2, d2, k2, p2[:, :1], g2[:, :1], R)
    ai[1::7, R // 2:] = -1  # some queries with fewer than R initial candidates
    ad[1::7, R // 2:] = np.inf
    tau = ad[:, R - 1].copy()
    tau[::5] = np.inf  # some queries unseeded
    t0 = torch.from_numpy(tau).cuda()
    ti, td = torch.from_numpy(ai).cuda(), torch.from_numpy(ad).cuda()
    pb, gb = probes[:, 1:], g[:, 1:]  # strided views: row stride nprobe
    for slices in (1, 2):
        for with_init in (False, True):
            ids = torch.empty((nq, R), dtype=torch.int64, device="cuda")
            dist = torch.empty((nq, R), dtype=torch.float32, device="cuda")
            init = (ptr(ti), ptr(td)) if with_init else (None, None)
            call("rbq_scan", idx.handle, ptr(qr), ptr(planes), ptr(delta), ptr(k1), nq, ptr(pb), ptr(gb),
                 nprobe - 1, nprobe, ptr(t0), *init, R, 1, slices, 0, ptr(ids), ptr(dist), None, 4, stream())
            oi, od = oracle.scan(oix, Qr, pl2, d2, k2, p2[:, 1:], g2[:, 1:], R, prune=1, slices=slices, tau0=tau,
                                 init=(ai, ad) if with_init else None)
            assert np.array_equal(ids.cpu().numpy(), oi)
            assert np.array_equal(u32(dist.cpu().numpy()), u32(od))


def test_balanced_shards_follow_the_restated_map(oracle, case, tmp_path):
    """RBQ_SHARD_BALANCED: the map fixed at the first add equals the oracle's restatement, each
    shard holds exactly its lists and searches them bit-exactly; the map survives save / load,
    and a full index loaded as one shard derives the same map from its list sizes."""
    from neurosamble_b200 import IndexIVFRaBitQ, read_index, write_index
    idx, oix, X, Q, C, lab = case
    sizes = np.bincount(lab, minlength=64)
    want = oracle.list_owners("balanced", sizes, 3)
    assert np.array_equal(oracle.list_owners("round_robin", sizes, 3), np.arange(64) % 3)
    for r in range(3):
        sh = IndexIVFRaBitQ(128, 64, seed=7, shard_rank=r, shard_count=3, shard_policy="balanced")
        assert (sh.list_owners() == -1).all()
        sh.set_centroids(C)
        sh.add(X, labels=lab)
        assert np.array_equal(sh.list_owners(), want)
        sz = np.diff(sh.export_lists()["list_off"])
        assert np.array_equal(sz[want == r], sizes[want == r]) and (sz[want != r] == 0).all()
        sh.nprobe, sh.k_rerank = 8, 40
        d, i = sh.search(Q, 10)
        d2, i2 = oracle.search(oix, Q, 10, 8, 40, shard_rank=r, shard_count=3, owner=want)
        assert np.array_equal(i, i2) and np.array_equal(u32(d), u32(d2))
        path = tmp_path / f"s{r}.rbq"
        write_index(sh, str(path))
        assert np.array_equal(read_index(str(path)).list_owners(), want)
    full = IndexIVFRaBitQ(128, 64, seed=7, shard_policy="balanced")
    full.set_centroids(C)
    full.add(X, labels=lab)
    assert (full.list_owners() == 0).all()
    path = tmp_path / "full.rbq"
    write_index(full, str(path))
    assert np.array_equal(read_index(str(path), shard_rank=1, shard_count=3).list_owners(), want)


@pytest.mark.parametrize("parts,k,sorted_rows", [(2, 10, 0), (8, 10, 0), (3, 40, 0), (8, 30, 0), (8, 100, 0),
                                                (8, 100, 1), (3, 40, 1), (5, 64, 1)])
def test_merge_results_matches_oracle(oracle, parts, k, sorted_rows):
    """rbq_merge_results ([parts, nq, k] -> [nq, k] by (distance, id)): the warp path for small
    merges; for large ones the rank merge of ascending rows (what shards return) and the block
    sort of unordered ones; with empty slots and a key present in two parts."""
    torch = _torch()
    rng = np.random.default_rng(parts * 1000 + k)
    nq = 77
    d = rng.standard_normal((parts, nq, k)).astype(np.float32)
    i = rng.integers(0, 1 << 31, (parts, nq, k)).astype(np.int64)
    i[:, ::3, k // 2:] = -1
    d[:, ::3, k // 2:] = np.inf
    d[0, 1, 0], i[0, 1, 0] = d[parts - 1, 1, 1], i[parts - 1, 1, 1]  # duplicate key
    if sorted_rows:  # each part's row ascending by key, as a search returns it
        order = np.argsort(oracle._keys(i, d), axis=2, kind="stable")
        d, i = np.take_along_axis(d, order, 2), np.take_along_axis(i, order, 2)
    od = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    oi = torch.empty((nq, k), dtype=torch.int64, device="cuda")
    dd, ii = torch.from_numpy(d).cuda(), torch.from_numpy(i).cuda()
    call("rbq_merge_results", ptr(dd), ptr(ii), parts, nq, k, ptr(od), ptr(oi), stream())
    wi, wd = oracle.merge_candidates([(i[p], d[p]) for p in range(parts)], k)
    assert np.array_equal(oi.cpu().numpy(), wi)
    assert np.array_equal(u32(od.cpu().numpy()), u32(wd))
    # the same merge from 8-byte result keys (what a sharded search all-gathers)
    keys = torch.empty((parts, nq, k), dtype=torch.int64, device="cuda")
    call("rbq_pack_results", ptr(dd), ptr(ii), parts * nq * k, ptr(keys), stream())
    assert np.array_equal(keys.cpu().numpy().view(np.uint64), oracle._keys(i, d))
    call("rbq_merge_result_keys", ptr(keys), parts, nq, k, ptr(od), ptr(oi), stream())
    assert np.array_equal(oi.cpu().numpy(), wi)
    assert np.array_equal(u32(od.cpu().numpy()), u32(wd))


@pytest.mark.parametrize("nprobe,R", [(1, 30), (1, 400), (5, 100)])
def test_bound_seed_matches_oracle(oracle, case, nprobe, R):
    """rbq_bound_seed: the R-th smallest upper bound over the leading whole lists holding >= R
    vectors (+inf when the probes hold fewer), bit-exact; also on a shard, where a query whose
    nearest list lives elsewhere gets +inf."""
    torch = _torch()
    idx, oix, X, Q, C, lab = case
    nq = Q.shape[0]
    Qr = oracle.rotate(Q, oix.P)
    qr, planes, delta, k1 = _query_stage(idx, Qr)
    P = 12
    probes = torch.empty((nq, P), dtype=torch.int32, device="cuda")
    g = torch.empty((nq, P), dtype=torch.float32, device="cuda")
    call("rbq_coarse", idx.handle, ptr(qr), nq, P, 0, ptr(probes), ptr(g), stream())
    p2, g2 = oracle.coarse(Qr, oix.c_rot, P)
    pl2, d2, k2, _ = oracle.query_prep(Qr, oix.t4)
    tau = torch.empty(nq, dtype=torch.float32, device="cuda")
    call("rbq_bound_seed", idx.handle, ptr(qr), ptr(planes), ptr(delta), ptr(k1), nq, ptr(probes), ptr(g), nprobe, P,
         R, 0, ptr(tau), 4, stream())
    want = oracle.bound_seed(oix, pl2, d2, k2, p2[:, :nprobe], g2[:, :nprobe], R)
    got = tau.cpu().numpy()
    assert np.array_equal(u32(got), u32(want))
    assert np.isfinite(want).any() and (R < 300 or np.isinf(want).any())


@pytest.mark.parametrize("n,d,K,iters,mtp", [(8000, 32, 24, 6, 256), (8000, 64, 48, 10, 64), (3000, 100, 7, 3, 256)])
def test_gpu_balanced_kmeans_matches_oracle(oracle, n, d, K, iters, mtp):
    """rbq_train (RBQ_KMEANS_BALANCED) vs the oracle's restatement of the reference's
    hierarchical balanced k-means on the same strided sample: centroids bit-exact."""
    from neurosamble_b200 import IndexIVFRaBitQ
    rng = np.random.default_rng(K)
    cen = rng.normal(size=(40, d)).astype(np.float32)
    w = 1.0 / np.arange(1, 41)
    X = (cen[rng.choice(40, size=n, p=w / w.sum())] + 0.3 * rng.normal(size=(n, d))).astype(np.float32)
    idx = IndexIVFRaBitQ(d, K, seed=5, kmeans_iters=iters, max_train_points_per_cluster=mtp)
    assert idx.info().kmeans_kind == 0
    idx.train(X)
    C = idx.centroids()[0]
    C2 = oracle.kmeans_balanced(oracle.train_sample(X, K, mtp), K, iters=iters)
    assert np.array_equal(u32(C), u32(C2))


def test_gpu_lloyd_kmeans_matches_oracle(oracle):
    """RBQ_KMEANS_LLOYD vs the oracle's Lloyd iterations: centroids bit-exact."""
    from neurosamble_b200 import IndexIVFRaBitQ
    X, _ = mixture(6000, 64, 30, 0.3, 1, seed=4)
    idx = IndexIVFRaBitQ(64, 20, seed=5, kmeans_iters=4, kmeans="lloyd")
    assert idx.info().kmeans_kind == 1
    idx.train(X)
    C2, _ = oracle.kmeans(oracle.train_sample(X, 20), 20, iters=4)
    assert np.array_equal(u32(idx.centroids()[0]), u32(C2))


def test_search_front_end_subchunks_equal_small_batches(oracle):
    """K = 8192: the coarse front end of a 40,000-query search runs in three [16384, K] score
    sub-chunks under one scan (and the long-row top-m path); the probes equal the oracle's and
    the results equal the same queries searched 5,000 at a time."""
    from neurosamble_b200 import IndexIVFRaBitQ
    X, Q = mixture(60000, 32, 500, 0.3, 40000, seed=9)
    K = 8192
    idx = IndexIVFRaBitQ(32, K, seed=2)
    C = np.ascontiguousarray(X[::7][:K])
    idx.set_centroids(C)
    idx.add(X)
    torch = _torch()
    nq, P = 400, 8
    dp = idx.info().padded_dim
    qr = torch.empty((nq, dp), dtype=torch.float32, device="cuda")
    q = dev(Q[:nq])
    call("rbq_rotate", idx.handle, ptr(q), nq, ptr(qr), stream())
    probes = torch.empty((nq, P), dtype=torch.int32, device="cuda")
    g = torch.empty((nq, P), dtype=torch.float32, device="cuda")
    call("rbq_coarse", idx.handle, ptr(qr), nq, P, 0, ptr(probes), ptr(g), stream())
    torch.cuda.synchronize()
    p2, g2 = oracle.coarse(qr.cpu().numpy(), idx.centroids()[1], P)
    assert np.array_equal(probes.cpu().numpy(), p2) and np.array_equal(u32(g.cpu().numpy()), u32(g2))
    # one scan kind for both batch sizes (auto would take the list scan for 40,000 queries and
    # the tile scan for 5,000, whose thresholds differ)
    idx.nprobe, idx.k_rerank, idx.scan_kind = P, 20, 1
    d, i = idx.search(Q, 10)
    parts = [idx.search(Q[a:a + 5000], 10) for a in range(0, 40000, 5000)]
    assert np.array_equal(i, np.concatenate([p[1] for p in parts]))
    assert np.array_equal(u32(d), u32(np.concatenate([p[0] for p in parts])))


def test_build_equals_train_or_centroids_then_add(oracle):
    """rbq_build (ivf_rabitq::build): with centroids it equals set_centroids + add, without
    them train + add (same lists, ids, codes); labels need the centroids they refer to."""
    from neurosamble_b200 import IndexIVFRaBitQ
    X, _ = mixture(6000, 64, 30, 0.3, 1, seed=12)
    a = IndexIVFRaBitQ(64, 24, seed=4, kmeans_iters=3)
    a.build(X)
    b = IndexIVFRaBitQ(64, 24, seed=4, kmeans_iters=3)
    b.train(X)
    b.add(X)
    ea, eb = a.export_lists(), b.export_lists()
    assert all(np.array_equal(ea[key], eb[key]) for key in ("list_off", "ids", "codes"))
    C = b.centroids()[0]
    lab = oracle.assign(X, C)
    c = IndexIVFRaBitQ(64, 24, seed=4)
    c.build(X, centroids=C, labels=lab)
    ec = c.export_lists()
    assert all(np.array_equal(ec[key], eb[key]) for key in ("list_off", "ids", "codes"))
    d = IndexIVFRaBitQ(64, 24, seed=4)
    with pytest.raises(RuntimeError, match="labels need the centroids"):
        d.build(X, labels=lab)
    with pytest.raises(RuntimeError, match="already holds"):
        c.build(X, centroids=C)


def test_injected_allocation_failure_is_reported_and_leaves_the_index_usable():
    """Out-of-memory handling without exhausting the shared GPU: rbq_debug_fail_alloc makes one
    device allocation fail as cudaMalloc would; the call returns RBQ_ERR_OOM (RuntimeError),
    the next call succeeds with the same results, and a failed create leaves no handle."""
    from neurosamble_b200 import IndexIVFRaBitQ, _lib
    L = _lib.lib()
    X, Q = mixture(8000, 64, 30, 0.3, 300, seed=13)
    idx = IndexIVFRaBitQ(64, 32, seed=4, kmeans_iters=3)
    idx.build(X)
    idx.nprobe, idx.k_rerank = 8, 30
    d0, i0 = idx.search(Q, 10)
    try:
        for after in (0, 1, 3):
            assert L.rbq_debug_fail_alloc(after) == 0
            with pytest.raises(RuntimeError, match="out of device memory.*injected"):
                idx.search(Q, 10)
            d1, i1 = idx.search(Q, 10)  # one shot: the hook is off again
            assert np.array_equal(i1, i0) and np.array_equal(u32(d1), u32(d0))
        L.rbq_debug_fail_alloc(0)
        with pytest.raises(RuntimeError, match="out of device memory"):
            IndexIVFRaBitQ(64, 16, seed=1)
    finally:
        L.rbq_debug_fail_alloc(-1)


def test_search_is_deterministic_run_to_run():
    """The same batch searched twice (single pass and split into slices) gives identical bits."""
    from neurosamble_b200 import IndexIVFRaBitQ
    X, Q = mixture(20000, 128, 50, 0.3, 257, seed=14)
    idx = IndexIVFRaBitQ(128, 64, seed=4, kmeans_iters=3)
    idx.build(X)
    idx.nprobe, idx.k_rerank = 12, 50
    for split in (0, 4):
        idx.probe_split = split
        a = idx.search(Q, 10)
        b = idx.search(Q, 10)
        assert np.array_equal(a[1], b[1]) and np.array_equal(u32(a[0]), u32(b[0]))



# ---- QUANT8 (search_mode::QUANT8: 8-bit query codes, scale t8 = best rescale for 7 extra bits)
def test_quant8_query_planes_bit_exact(oracle, case):
    idx, oix, X, Q, C, lab = case
    Qr = oracle.rotate(Q, oix.P)
    _, planes, delta, k1 = _query_stage(idx, Qr, 8)
    p2, d2, k2, codes = oracle.query_prep(Qr, oracle.query_scale(128, 7, 7), 8)
    assert planes.shape[1] == 8 and np.array_equal(u32(planes.cpu().numpy()), p2)
    assert np.array_equal(u32(delta.cpu().numpy()), u32(d2)) and np.array_equal(u32(k1.cpu().numpy()), u32(k2))
    assert codes.min() < -8 or codes.max() > 7  # the 8-bit range is used


@pytest.mark.parametrize("prune,slices,R", [(1, 1, 40), (0, 1, 40), (1, 4, 40), (1, 1, 100)])
def test_quant8_scan_candidates_bit_exact(oracle, case, prune, slices, R):
    idx, oix, X, Q, C, lab = case
    gi, gd, gst, oi, od, ost = _scan(idx, oracle, oix, Q, 8, R, prune, slices, 0, bits=8)
    assert np.array_equal(gi, oi) and np.array_equal(u32(gd), u32(od))
    assert gst.tolist() == ost.tolist()


@pytest.mark.parametrize("nprobe,R,seeded", [(8, 40, -1), (16, 40, 1), (4, 0, 0)])
def test_quant8_search_end_to_end(oracle, case, nprobe, R, seeded):
    idx, oix, X, Q, C, lab = case
    oix.t8 = oracle.query_scale(128, 7, 7)
    idx.nprobe, idx.k_rerank, idx.prune, idx.seeded, idx.query_bits = nprobe, R, True, seeded, 8
    try:
        d, i = idx.search(Q, 10)
    finally:
        idx.query_bits, idx.seeded = 4, -1
    d2, i2 = oracle.search(oix, Q, 10, nprobe, R, prune=1, seeded=seeded, query_bits=8)
    assert np.array_equal(i, i2) and np.array_equal(u32(d), u32(d2))
    if R:
        d4, i4 = oracle.search(oix, Q, 10, nprobe, R, prune=1, seeded=seeded)
        _, gt = oracle.knn_exact(X, Q, 10)
        assert oracle.recall(i, gt) >= oracle.recall(i4, gt) - 0.02


def test_quant8_stage_ops_compose_to_the_search(case):
    torch = _torch()
    idx, oix, X, Q, C, lab = case
    h, P, R, k = idx.handle.value, 8, 40, 10
    q = dev(Q)
    ops = torch.ops.rbq
    qr = ops.rotate(h, q)
    probes, g = ops.coarse(h, qr, P, 0)
    planes, delta, k1 = ops.query_prep(h, qr, 8)
    cand, _ = ops.scan(h, qr, planes, delta, k1, probes, g, R, True, 1, 0, None)
    d, i = ops.rerank(h, q, cand, k)
    d2, i2 = ops.search(h, q, k, P, R, True, 1, 0, 8)
    torch.cuda.synchronize()
    assert torch.equal(i, i2) and np.array_equal(u32(d.cpu().numpy()), u32(d2.cpu().numpy()))


def test_query_bits_are_checked(case):
    idx, oix, X, Q, C, lab = case
    idx.query_bits = 5
    try:
        with pytest.raises(RuntimeError, match="QUANT4.*QUANT8"):
            idx.search(Q[:3], 5)
    finally:
        idx.query_bits = 4


@pytest.mark.parametrize("mode", [16, 32])
@pytest.mark.parametrize("slices,R", [(1, 40), (3, 100)])
def test_lut_scan_candidates_bit_exact(oracle, case, mode, slices, R):
    """LUT16 / LUT32 (computeInnerProductsWithLUT16Opt): the scan's candidates are the top R by
    the table estimate, bit for bit the oracle's tables (fp16 rounding included) and sums."""
    torch = _torch()
    idx, oix, X, Q, C, lab = case
    Qr = oracle.rotate(Q, oix.P)
    nq, nprobe = Qr.shape[0], 8
    qr, planes, delta, k1 = _query_stage(idx, Qr, 4)
    probes = torch.empty((nq, nprobe), dtype=torch.int32, device="cuda")
    g = torch.empty((nq, nprobe), dtype=torch.float32, device="cuda")
    call("rbq_coarse", idx.handle, ptr(qr), nq, nprobe, 0, ptr(probes), ptr(g), stream())
    ids = torch.empty((nq, R), dtype=torch.int64, device="cuda")
    dist = torch.empty((nq, R), dtype=torch.float32, device="cuda")
    stats = torch.zeros(2, dtype=torch.int64, device="cuda")
    call("rbq_scan", idx.handle, ptr(qr), ptr(planes), ptr(delta), ptr(k1), nq, ptr(probes), ptr(g), nprobe, 0, None,
         None, None, R, 1, slices, 0, ptr(ids), ptr(dist), ptr(stats), mode, stream())
    p2, g2 = oracle.coarse(Qr, oix.c_rot, nprobe)
    pl2, d2, k2, _ = oracle.query_prep(Qr, oix.t4, 4)
    oi, od, ost = oracle.scan(oix, Qr, pl2, d2, k2, p2, g2, R, slices=slices, with_stats=True, mode=mode)
    assert np.array_equal(ids.cpu().numpy(), oi)
    assert np.array_equal(u32(dist.cpu().numpy()), u32(od))
    assert stats.cpu().tolist() == ost.tolist()


@pytest.mark.parametrize("mode", [16, 32])
@pytest.mark.parametrize("R", [0, 40])
def test_lut_search_end_to_end(oracle, case, mode, R):
    """The LUT16 / LUT32 search (estimates returned as they are with R = 0, as the reference
    does, or reranked exactly) equals the oracle's, for one and several probe slices."""
    idx, oix, X, Q, C, lab = case
    idx.nprobe, idx.k_rerank, idx.prune, idx.seeded, idx.query_bits = 8, R, True, -1, mode
    try:
        for qs in (Q, Q[:5]):
            d, i = idx.search(qs, 10)
            sl = max(1, min(512 // len(qs), 8)) if len(qs) < 512 else 1
            d2, i2 = oracle.search(oix, qs, 10, 8, R, slices=sl, query_bits=mode)
            assert np.array_equal(i, i2) and np.array_equal(u32(d), u32(d2))
    finally:
        idx.query_bits = 4


def test_host_raw_store_gives_the_device_store_results(oracle, tmp_path):
    """raw_store="host": the raw rows live in pinned host memory (the rerank reads them over
    PCIe) so only codes, factors and ids need HBM.  Built in several adds, the index searches,
    saves and reloads bit-equal to the same index with its rows in HBM."""
    from neurosamble_b200 import IndexIVFRaBitQ, read_index, write_index
    X, Q = mixture(12000, 96, 30, 0.3, 150, seed=41)
    res = []
    for store in ("device", "host"):
        idx = IndexIVFRaBitQ(96, 48, seed=7, kmeans_iters=4, raw_store=store)
        idx.train(X)
        for a in range(0, len(X), 5000):
            idx.add(X[a:a + 5000])
        idx.nprobe, idx.k_rerank = 12, 60
        res.append(idx.search(Q, 10))
        if store == "host":
            write_index(idx, str(tmp_path / "h.rbq"))
            back = read_index(str(tmp_path / "h.rbq"))
            back.nprobe, back.k_rerank = 12, 60
            res.append(back.search(Q, 10))
    for d, i in res[1:]:
        assert np.array_equal(i, res[0][1]) and np.array_equal(u32(d), u32(res[0][0]))
    C, _ = idx.centroids()
    oix = oracle.build(X, C, oracle.assign(X, C), idx.rotation(), idx.query_scale)
    d2, i2 = oracle.search(oix, Q, 10, 12, 60)
    assert np.array_equal(res[0][1], i2) and np.array_equal(u32(res[0][0]), u32(d2))


def test_graph_search_replays_bit_exact(case):
    """use_graph: the first search of a batch size is captured as a CUDA graph, later ones
    replay it (new inputs copied in, results copied out); a replay launches no kernel of its
    own and returns the bits of a plain search, on the device and the host-buffer paths."""
    import ctypes
    torch = _torch()
    from neurosamble_b200 import _lib
    idx, oix, X, Q, C, lab = case
    idx.nprobe, idx.k_rerank, idx.prune, idx.seeded = 8, 40, True, -1
    L = _lib.lib()
    try:
        for B in (1, 7, 64):
            idx.use_graph = False
            want = [idx.search(Q[a:a + B], 10) for a in (0, B, 2 * B)]
            idx.use_graph = True
            got = [idx.search(Q[a:a + B], 10) for a in (0, B, 2 * B)]
            for (d0, i0), (d1, i1) in zip(want, got):
                assert np.array_equal(i0, i1) and np.array_equal(u32(d0), u32(d1))
            n0 = L.rbq_kernel_launches()
            d2, i2 = idx.search(Q[B:2 * B], 10)
            assert L.rbq_kernel_launches() == n0  # a replay: no kernels launched one by one
            assert np.array_equal(i2, want[1][1])
            sp = idx.search_params(10)
            dh = np.empty((B, 10), np.float32)
            ih = np.empty((B, 10), np.int64)
            qh = np.ascontiguousarray(Q[2 * B:3 * B])
            call("rbq_search_host", idx.handle, ctypes.byref(sp), qh.ctypes.data_as(ctypes.c_void_p), B,
                 dh.ctypes.data_as(ctypes.c_void_p), ih.ctypes.data_as(ctypes.c_void_p), stream())
            assert np.array_equal(ih, want[2][1]) and np.array_equal(u32(dh), u32(want[2][0]))
    finally:
        idx.use_graph = False
    torch.cuda.synchronize()


def test_graph_replays_on_two_streams_do_not_share_results(case):
    """Replays of one captured search issued back to back on two streams (no sync between):
    each stream must get its own batch's results, bit-equal to plain searches, although the
    graph's input and output buffers are shared."""
    torch = _torch()
    from neurosamble_b200 import _lib
    idx, oix, X, Q, C, lab = case
    idx.nprobe, idx.k_rerank, idx.prune, idx.seeded = 8, 40, True, -1
    B = 64
    batches = [dev(Q[a:a + B]) for a in range(0, 4 * B, B)]
    idx.use_graph = False
    want = [idx.search(Q[a:a + B], 10) for a in range(0, 4 * B, B)]
    sp = idx.search_params(10)
    sp.graph = 1
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [(torch.empty((B, 10), dtype=torch.float32, device="cuda"),
             torch.empty((B, 10), dtype=torch.int64, device="cuda")) for _ in batches]
    try:
        call("rbq_search", idx.handle, ctypes.byref(sp), ptr(batches[0]), B, ptr(outs[0][0]), ptr(outs[0][1]),
             stream())  # captures the graph
        for rep in range(3):
            for j, qb in enumerate(batches):
                st = streams[j % 2]
                _lib.call("rbq_search", idx.handle, ctypes.byref(sp), ptr(qb), B, ptr(outs[j][0]), ptr(outs[j][1]),
                       ctypes.c_void_p(st.cuda_stream))
            torch.cuda.synchronize()
            for (d0, i0), (d1, i1) in zip(want, outs):
                assert np.array_equal(i0, i1.cpu().numpy()) and np.array_equal(u32(d0), u32(d1.cpu().numpy()))
    finally:
        idx.use_graph = False
    torch.cuda.synchronize()


def test_graphs_are_dropped_when_the_index_changes(oracle):
    from neurosamble_b200 import IndexIVFRaBitQ
    X, Q = mixture(8000, 64, 30, 0.3, 16, seed=15)
    idx = IndexIVFRaBitQ(64, 16, seed=4, kmeans_iters=3)
    idx.build(X[:5000])
    idx.nprobe, idx.k_rerank, idx.use_graph = 4, 20, True
    d1, i1 = idx.search(Q, 5)
    idx.add(X[5000:])  # reallocates the lists: the captured search must not be replayed
    d2, i2 = idx.search(Q, 5)
    idx.use_graph = False
    d3, i3 = idx.search(Q, 5)
    assert np.array_equal(i2, i3) and np.array_equal(u32(d2), u32(d3))
    assert (i3 >= 5000).any() and not (i1 >= 5000).any()
