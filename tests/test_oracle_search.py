"""Properties of the oracle's search schedule (CPU): the facts the GPU parity tests rely on."""
import numpy as np
import pytest

from conftest import mixture


def build_small(oracle, n=6000, d=64, k=32, nq=40, seed=0, dp_seed=11):
    X, Q = mixture(n, d, 24, 0.3, nq, seed=seed)
    P = oracle.make_rotation(oracle.pad_dim(d), dp_seed)
    t4 = oracle.query_scale(oracle.pad_dim(d), dp_seed)
    C, lab = oracle.kmeans(X, k, iters=4)
    return oracle.build(X, C, lab, P, t4), X, Q, lab


@pytest.fixture(scope="module")
def small(oracle):
    return build_small(oracle)


def prep(oracle, ix, Q, nprobe):
    Qr = oracle.rotate(Q, ix.P)
    probes, g = oracle.coarse(Qr, ix.c_rot, nprobe)
    planes, delta, k1, _ = oracle.query_prep(Qr, ix.t4)
    return Qr, probes, g, planes, delta, k1


def test_layout_is_stable_counting_sort(oracle, small):
    ix, X, Q, lab = small
    assert ix.list_off[0] == 0 and ix.list_off[-1] == X.shape[0]
    for l in range(ix.k):
        members = ix.ids[ix.list_off[l]:ix.list_off[l + 1]]
        assert np.all(lab[members] == l)
        assert np.all(np.diff(members.astype(np.int64)) > 0)


def test_exhaustive_scan_equals_estimator_sort(oracle, small):
    """nprobe = nlist, prune off: the scan's top-R is the plain sort of every estimate."""
    ix, X, Q, lab = small
    Qr, probes, g, planes, delta, k1 = prep(oracle, ix, Q[:5], ix.k)
    R = 30
    ids, dist = oracle.scan(ix, Qr, planes, delta, k1, probes, g, R, prune=0)
    W = ix.dp // 32
    for q in range(5):
        gl = {int(l): float(gv) for l, gv in zip(probes[q], g[q])}
        keys = []
        for l in range(ix.k):
            for s in range(ix.list_off[l], ix.list_off[l + 1]):
                eip = np.float32(oracle.exact_ip(Qr[q], ix.codes[s]))
                base = np.float32(ix.fadd[s]) + np.float32(gl[l])
                dd = base + np.float32(ix.frescale[s]) * (eip + np.float32(k1[q]))
                keys.append((float(np.float32(dd)), int(ix.ids[s])))
        keys.sort()
        assert [i for _, i in keys[:R]] == ids[q].tolist()
        assert np.array_equal(np.array([d for d, _ in keys[:R]], np.float32).view(np.uint32),
                              dist[q].view(np.uint32))


def test_no_prune_result_is_schedule_independent(oracle, small):
    ix, X, Q, lab = small
    Qr, probes, g, planes, delta, k1 = prep(oracle, ix, Q, 8)
    base = oracle.scan(ix, Qr, planes, delta, k1, probes, g, 20, prune=0)
    for tile, cap, slices in ((256, 512, 1), (256, 2048, 1), (128, 1024, 3), (256, 1024, 8)):
        other = oracle.scan(ix, Qr, planes, delta, k1, probes, g, 20, tile=tile, cap=cap, prune=0,
                            slices=slices)
        assert np.array_equal(base[0], other[0])


def test_prune_keeps_recall(oracle, small):
    ix, X, Q, lab = small
    _, gt = oracle.knn_exact(X, Q, 10)
    d0, i0 = oracle.search(ix, Q, 10, 8, 40, prune=0)
    d1, i1, st = oracle.search(ix, Q, 10, 8, 40, prune=1, with_stats=True)
    assert st[1] < st[0]  # the prune removes work
    assert abs(oracle.recall(i0, gt) - oracle.recall(i1, gt)) <= 0.01


def test_sharded_union_equals_unsharded_without_prune(oracle, small):
    ix, X, Q, lab = small
    Qr, probes, g, planes, delta, k1 = prep(oracle, ix, Q, 8)
    R = 25
    full = oracle.scan(ix, Qr, planes, delta, k1, probes, g, R, prune=0)
    parts = [oracle.scan(ix, Qr, planes, delta, k1, probes, g, R, prune=0, shard_rank=r, shard_count=3)
             for r in range(3)]
    for q in range(Q.shape[0]):
        keys = []
        for ids, dist in parts:
            keys += [(float(dist[q, j]), int(ids[q, j])) for j in range(R) if ids[q, j] >= 0]
        keys.sort()
        assert [i for _, i in keys[:R]] == full[0][q].tolist()


def test_rerank_returns_exact_order(oracle, small):
    ix, X, Q, lab = small
    cand = np.tile(np.arange(50, dtype=np.int64), (3, 1))
    cand[1, 10:] = -1
    d, i = oracle.rerank(X, Q[:3], cand, 10)
    for q in range(3):
        pool = [c for c in cand[q] if c >= 0]
        ref = sorted((oracle.l2_exact(X[c], Q[q]), c) for c in pool)[:10]
        assert i[q].tolist() == [c for _, c in ref]


def test_padding_when_fewer_candidates_than_k(oracle):
    ix, X, Q, lab = build_small(oracle, n=300, d=32, k=8, nq=3)
    d, i = oracle.search(ix, Q, 5, 1, 0, prune=1)
    assert np.all((i >= 0).sum(axis=1) >= 1)
    # one list only and huge k: the tail is padded
    d, i = oracle.search(ix, Q, 400, 1, 0, prune=0)
    assert (i == -1).any() and np.all(np.isinf(d[i == -1]))


def test_empty_lists_and_single_vector(oracle):
    X, Q = mixture(1, 32, 1, 0.3, 2, seed=4)
    P = oracle.make_rotation(32, 1)
    t4 = oracle.query_scale(32, 1)
    C = np.concatenate([X, X + 1.0, X - 1.0]).astype(np.float32)  # lists 1, 2 stay empty
    lab = np.zeros(1, np.uint32)
    ix = oracle.build(X, C, lab, P, t4)
    assert ix.list_off.tolist() == [0, 1, 1, 1]
    d, i = oracle.search(ix, Q, 3, 3, 0, prune=1)
    assert i[:, 0].tolist() == [0, 0] and np.all(i[:, 1:] == -1)


def test_reference_gtest_recall_floor(oracle):
    """cuVS gtest shape: 4096 x 64 U(0.1, 2), 1024 queries, k = 10, n_lists = clamp(N/128, 32,
    1024) = 32; 1-bit recall floor 0.3 (ann_ivf_rabitq.cuh:82-100, 218-230)."""
    rng = np.random.default_rng(1234)
    X = rng.uniform(0.1, 2.0, (4096, 64)).astype(np.float32)
    Q = rng.uniform(0.1, 2.0, (256, 64)).astype(np.float32)
    P = oracle.make_rotation(64, 7)
    t4 = oracle.query_scale(64, 7)
    C, lab = oracle.kmeans(X, 32, iters=6)
    ix = oracle.build(X, C, lab, P, t4)
    _, gt = oracle.knn_exact(X, Q, 10)
    _, ids = oracle.search(ix, Q, 10, 16, 0, prune=1)
    assert oracle.recall(ids, gt) >= 0.3


def test_seeded_scan_without_prune_is_the_plain_top_r(oracle, small):
    """A seed is the R-th estimate of a subset of the probed vectors, never below the true R-th:
    with the prune off the two-phase scan (any slicing, any shard count) keeps the exact top-R."""
    ix, X, Q, lab = small
    Qr, probes, g, planes, delta, k1 = prep(oracle, ix, Q, 8)
    R = 30
    full = oracle.scan(ix, Qr, planes, delta, k1, probes, g, R, prune=0)
    for slices in (1, 3):
        ids, dist = oracle.seeded_scan(ix, Qr, planes, delta, k1, probes, g, R, prune=0, slices=slices)
        assert np.array_equal(ids, full[0]) and np.array_equal(dist.view(np.uint32), full[1].view(np.uint32))
    parts = [oracle.seeded_scan(ix, Qr, planes, delta, k1, probes, g, R, prune=0, shard_rank=r, shard_count=3,
                                exchange=True) for r in range(3)]
    mi, md = oracle.merge_candidates(parts, R)
    assert np.array_equal(mi, full[0])


def test_seed_is_shared_and_keeps_shards_pruning(oracle, small):
    """exchange=True gives every shard the owner's phase-A threshold: the shards together admit
    about as many vectors as one shard (each shard's threshold then tightens only on its own
    candidates), far fewer than unseeded shards, which start from +inf."""
    ix, X, Q, lab = small
    Qr, probes, g, planes, delta, k1 = prep(oracle, ix, Q, 12)
    R = 40

    def admitted(shards, seeded):
        tot = np.zeros(2, np.int64)
        for r in range(shards):
            if seeded:
                st = oracle.seeded_scan(ix, Qr, planes, delta, k1, probes, g, R, shard_rank=r, shard_count=shards,
                                        with_stats=True, exchange=True)[2]
            else:
                st = oracle.scan(ix, Qr, planes, delta, k1, probes, g, R, shard_rank=r, shard_count=shards,
                                 with_stats=True)[2]
            tot += st
        return tot

    one, four = admitted(1, True), admitted(4, True)
    assert one[0] == four[0]  # every probed vector is scanned exactly once
    assert four[1] <= one[1] * 1.25
    assert admitted(4, False)[1] > 1.5 * four[1]
    # shard_count = 1: the exchanged seed is the shard's own
    a = oracle.seeded_scan(ix, Qr, planes, delta, k1, probes, g, R, exchange=True)
    b = oracle.seeded_scan(ix, Qr, planes, delta, k1, probes, g, R, exchange=False)
    assert np.array_equal(a[0], b[0])


def test_balanced_list_owners_restated(oracle):
    """The balanced map: every list placed, ties resolved by list id then rank, and no shard's
    sum of size^2 exceeds another's by more than the largest single size^2."""
    rng = np.random.default_rng(5)
    sizes = rng.integers(0, 3000, 300)
    sizes[:4] = [2500, 2500, 0, 0]
    for count in (1, 2, 3, 8):
        own = oracle.list_owners("balanced", sizes, count)
        assert own.shape == (300,) and own.min() >= 0 and own.max() < count
        load = np.bincount(own, weights=sizes.astype(np.float64) ** 2, minlength=count)
        assert load.max() - load.min() <= float(sizes.max()) ** 2
    assert oracle.list_owners("balanced", [5, 5, 3], 2).tolist() == [0, 1, 0]
    assert oracle.list_owners("balanced", [3, 5, 5], 2).tolist() == [0, 0, 1]


def _skewed(n=8000, d=32, nc=40, seed=0):
    rng = np.random.default_rng(seed)
    cen = rng.normal(size=(nc, d)).astype(np.float32)
    w = 1.0 / np.arange(1, nc + 1)
    a = rng.choice(nc, size=n, p=w / w.sum())
    X = (cen[a] + 0.3 * rng.normal(size=(n, d))).astype(np.float32)
    return X / np.linalg.norm(X, axis=1, keepdims=True)


def test_balanced_kmeans_restated(oracle):
    """Hierarchical balanced k-means (kmeans_balanced.cuh:759-1132) on a Zipf-skewed mixture:
    deterministic, every list non-empty, and the largest list smaller than plain Lloyd's."""
    X = _skewed()
    K = 48
    C1 = oracle.kmeans_balanced(X, K, iters=10)
    C2 = oracle.kmeans_balanced(X, K, iters=10)
    assert C1.dtype == np.float32 and C1.shape == (K, 32) and np.array_equal(C1, C2)
    sb = np.bincount(oracle.assign(X, C1), minlength=K)
    _, ll = oracle.kmeans(X, K, iters=10)
    sl = np.bincount(ll, minlength=K)
    assert sb.min() > 0 and sb.max() < sl.max()


def test_balanced_kmeans_pieces(oracle):
    """The rebalancing walk visits every row (its stride never divides n), a small cluster's
    centre moves to (wc * c_big + x) / (wc + 1) in float32, and an empty cluster's centre is
    zero after the M step."""
    from oracle.oracle import _km_adjust, _km_stride, _km_update
    for n in (1, 7, 61 * 67, 2 ** 20, 3 * 5 * 7 * 11 * 13 * 61):
        p = _km_stride([0], n)
        assert n % p != 0
    X = np.arange(12, dtype=np.float32).reshape(6, 2)
    lab = np.array([0, 0, 0, 0, 0, 1], np.uint32)
    C, size = _km_update(X, lab, 3, True, np.full((3, 2), 5, np.float32))
    assert size.tolist() == [5, 1, 0] and np.array_equal(C[2], [0, 0]) and np.array_equal(C[1], X[5])
    # limit = int((6 // 3) * 0.25) = 0: only the empty cluster 2 moves, towards the first row
    # of the walk whose cluster holds >= 2 rows; with wc = 0 it lands on that row.
    C2, moved = _km_adjust(X, C, lab, size, 0.25, [0])
    assert moved and np.array_equal(C2[:2], C[:2])
    i = _km_stride([0], 6) % 6
    assert lab[i] == 0 and np.array_equal(C2[2], X[i])
    # threshold 0.5: limit 1, cluster 1 (one row) moves too, with wc = 1 and the walk's next row
    C3, _ = _km_adjust(X, C, lab, size, 0.5, [0])
    st = _km_stride([0], 6)
    i1, i2 = st % 6, (2 * st) % 6
    w = np.float32(1)
    assert np.array_equal(C3[1], (np.float32(0) + w * C[0] + np.float32(1) * X[i1]) / (w + np.float32(1)))
    assert np.array_equal(C3[2], X[i2])



def test_quant8_planes_reconstruct_codes_and_tighten_the_estimate(oracle, small):
    """8-bit query codes (QUANT8): within [-128, 127], their two's-complement planes rebuild
    them, the popcount inner product equals sum code_j * bit_j, and acc * delta tracks the
    exact <q, bits> more closely than the 4-bit codes do."""
    ix = small[0]
    rng = np.random.default_rng(5)
    Q = rng.standard_normal((40, ix.d)).astype(np.float32)
    Qr = oracle.rotate(Q, ix.P)
    t8 = oracle.query_scale(ix.dp, 11, 7)
    p8, d8, k8, c8 = oracle.query_prep(Qr, t8, 8)
    p4, d4, k4, c4 = oracle.query_prep(Qr, ix.t4, 4)
    assert p8.shape[1] == 8 and c8.min() >= -128 and c8.max() <= 127 and np.abs(c8).max() > 7
    assert np.array_equal(k8, k4)
    w = ix.dp // 32
    bit = ((p8[:, :, :, None] >> (31 - np.arange(32, dtype=np.uint32))) & 1).transpose(0, 2, 3, 1)
    bit = bit.reshape(Q.shape[0], ix.dp, 8).astype(np.int64)
    rebuilt = (bit[:, :, :7] << np.arange(7)).sum(-1) - (bit[:, :, 7] << 7)
    assert np.array_equal(rebuilt, c8.astype(np.int64))
    err4 = err8 = 0.0
    for q in range(Q.shape[0]):
        for s in range(0, ix.codes.shape[0], 97):
            code = ix.codes[s]
            bits = ((code[:, None] >> (31 - np.arange(32, dtype=np.uint32))) & 1).reshape(-1).astype(np.int64)
            a8 = oracle.popcount_ip(p8[q], code)
            assert a8 == int((c8[q].astype(np.int64) * bits).sum())
            exact = float((Qr[q].astype(np.float64) * bits).sum())
            err8 += abs(a8 * float(d8[q]) - exact)
            err4 += abs(oracle.popcount_ip(p4[q], code) * float(d4[q]) - exact)
    assert err8 < 0.25 * err4


def test_query_scale_8bit_matches_the_library(oracle):
    """t8 (const_scaling_factor_8bit, best rescale with 7 extra bits) from the library's host
    math equals the oracle's restatement bit for bit."""
    import ctypes
    from neurosamble_b200 import _lib
    for dp in (32, 128, 256):
        t = ctypes.c_float()
        assert _lib.lib().rbq_query_scale(dp, 7, 7, ctypes.byref(t)) == 0
        assert np.float32(t.value).view(np.uint32) == np.float32(oracle.query_scale(dp, 7, 7)).view(np.uint32)


@pytest.mark.parametrize("n,K,iters", [(50, 1, 5), (16, 16, 5), (17, 16, 3), (100, 99, 2), (300, 40, 0), (1000, 3, 20)])
def test_balanced_kmeans_edge_cases(oracle, n, K, iters):
    """One list, as many lists as rows, zero iterations, mesoclusters with fewer rows than
    their share of fine clusters: finite centres, every list non-empty."""
    X = np.random.default_rng(n * K).standard_normal((n, 8)).astype(np.float32)
    C = oracle.kmeans_balanced(X, K, iters)
    assert C.shape == (K, 8) and np.isfinite(C).all()
    assert (np.bincount(oracle.assign(X, C), minlength=K) > 0).all()


def test_fp16_rounding_of_the_lut16_tables():
    """LUT16 rounds its table entries to fp16 as CUDA's __float2half does (nearest, ties to even);
    the oracle's own conversion must agree with IEEE (numpy) on normal, subnormal, halfway,
    overflow and special values, and convert back exactly."""
    from oracle import oracle as O
    rng = np.random.default_rng(0)
    hv = np.arange(0, 1 << 15, dtype=np.uint16).view(np.float16).astype(np.float32)
    hv = hv[np.isfinite(hv)]
    xs = np.concatenate([
        rng.standard_normal(100000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 6, 100000).astype(np.float32),
        np.arange(1, 4000, dtype=np.float32) * np.float32(2.0 ** -25),
        hv, ((hv[:-1] + hv[1:]) / 2).astype(np.float32), -hv,
        np.array([0.0, -0.0, 65504, 65519.99, 65520, 1e9, -1e9, np.inf, -np.inf], np.float32)])
    with np.errstate(over="ignore"):
        want = xs.astype(np.float16).view(np.uint16)
    got = O.float_to_half_bits(xs)
    assert np.array_equal(got, want)
    back = O.half_bits_to_float(got)
    assert np.array_equal(back.view(np.uint32), got.view(np.float16).astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("mode", [16, 32])
def test_lut_modes_rank_by_the_table_estimate(mode):
    """LUT16 / LUT32 return the top k by the table estimate with R = 0: with one slice and with
    several (each slice keeps its own top k, merged), and the same set as scoring every probed
    vector with the tables and sorting."""
    from conftest import mixture
    from oracle import oracle as O
    X, Q = mixture(5000, 64, 12, 0.3, 20, seed=3)
    P, t4 = O.make_rotation(64, 3), O.query_scale(64, 3)
    C, lab = O.kmeans(X, 16, iters=3)
    ix = O.build(X, C, lab, P, t4)
    d1, i1 = O.search(ix, Q, 10, 6, 0, query_bits=mode)
    d3, i3 = O.search(ix, Q, 10, 6, 0, query_bits=mode, slices=3)
    assert np.array_equal(i1, i3) and np.array_equal(d1.view(np.uint32), d3.view(np.uint32))
    assert np.all(np.diff(d1, axis=1) >= 0)
    _, gt = O.knn_exact(X, Q, 10)
    assert O.recall(i1, gt) > 0.3
