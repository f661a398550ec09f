"""The list scan (rbq_search_params_t.scan_kind = 2): fixed per-query thresholds and a tensor-core
int8 GEMM per probed list (query codes x code bits), then the exact pass per query.

Its result is defined by the oracle's `list_scan`: admit while low < tau0 (the bound seed over
the leading probed lists holding >= R vectors), keep the admitted vectors with distance <= tau0,
return the R smallest keys.  CPU tests pin that definition against the tile scan; GPU tests
compare the library with it bit for bit."""
import numpy as np
import pytest

from conftest import mixture


def u32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ------------------------------------------------------------------------------------------
# CPU: the definition
# ------------------------------------------------------------------------------------------
@pytest.fixture(scope="module")
def small(oracle):
    X, Q = mixture(30000, 128, 60, 0.3, 200, seed=21)
    C, _ = oracle.kmeans(X[::5], 48, iters=4)
    lab = oracle.assign(X, C)
    P, t4 = oracle.make_rotation(128, 7), oracle.query_scale(128, 7)
    return oracle.build(X, C, lab, P, t4), X, Q


def test_fixed_threshold_keeps_the_tile_scan_answer(oracle, small):
    """With thresholds fixed at the bound seed the admitted set contains the tile scan's (whose
    threshold only tightens from that seed), and the top R agree on this data."""
    ix, X, Q = small
    Qr = oracle.rotate(Q, ix.P)
    probes, g = oracle.coarse(Qr, ix.c_rot, 8)
    pl, de, k1, _ = oracle.query_prep(Qr, ix.t4, 4)
    R = 40
    tau = oracle.bound_seed(ix, pl, de, k1, probes, g, R)
    assert np.isfinite(tau).all()
    ti, td, ts = oracle.scan(ix, Qr, pl, de, k1, probes, g, R, with_stats=True, tau0=tau)
    li, ld, ls = oracle.list_scan(ix, Qr, pl, de, k1, probes, g, R, tau, with_stats=True)
    assert ls[0] == ts[0] and ls[1] >= ts[1]
    assert np.array_equal(li, ti) and np.array_equal(u32(ld), u32(td))


def test_auto_rule():
    from oracle import oracle as O
    assert O.uses_list_scan(0, 4, 1, 256, 10000, 32, 1024)      # 312 queries per list
    assert O.uses_list_scan(0, 4, 1, 256, 10000, 32, 1024, 1_000_000, 200)  # lists of 976 >= R
    assert not O.uses_list_scan(0, 4, 1, 256, 200000, 48, 2048, 200_000, 800)  # lists of 98 < R
    assert not O.uses_list_scan(0, 4, 1, 256, 64, 32, 1024)     # 2 per list: the tile scan
    assert not O.uses_list_scan(0, 16, 1, 256, 10000, 32, 1024)  # LUT modes scan by tiles
    assert not O.uses_list_scan(0, 4, 0, 256, 10000, 32, 1024)   # no prune: nothing to fix
    assert not O.uses_list_scan(1, 4, 1, 256, 10000, 32, 1024)
    assert O.uses_list_scan(2, 8, 1, 768, 1, 1, 1024)
    with pytest.raises(ValueError):
        O.uses_list_scan(2, 4, 1, 1024, 1, 1, 8)


def test_word_to_vector_mapping_by_multiply_high():
    """The list scan maps its code-word index i (< N * 24, N = 128 vectors per tile) to the vector
    i / W by a multiply-high with ceil(2^32 / W) instead of an integer division: exact for every
    word count W = Dp / 32 up to 24 (Dp <= 768) over that whole range."""
    i = np.arange(128 * 24 + 1, dtype=np.uint64)
    for W in range(1, 25):
        magic = np.uint64((2 ** 32 + W - 1) // W)
        assert np.array_equal((i * magic) >> np.uint64(32), i // np.uint64(W)), W


@pytest.mark.parametrize("QB", [4, 8])
@pytest.mark.parametrize("W", [1, 2, 4, 8, 24])
def test_int8_gemm_form_equals_the_popcount_estimator(oracle, QB, W):
    """The list scan's A operand: a query's planes read back as signed int8 codes (two's
    complement over its QB planes, bit j of a plane word's reversal = dim j).  The int8 dot product
    of those codes with a vector's code bits is the popcount estimator's integer, for any planes."""
    rng = np.random.default_rng(QB * 100 + W)
    for _ in range(30):
        planes = rng.integers(0, 2 ** 32, (QB, W), dtype=np.uint64).astype(np.uint32)
        code = rng.integers(0, 2 ** 32, W, dtype=np.uint64).astype(np.uint32)
        dims = np.arange(32 * W)
        w, j = dims // 32, dims % 32
        pbits = (planes[:, w].astype(np.int64) >> (31 - j)) & 1  # [QB, dims]: plane b, dim 32w + j
        q8 = sum(pbits[b] << b for b in range(QB - 1)) - (pbits[QB - 1] << (QB - 1))
        assert q8.min() >= -(1 << (QB - 1)) and q8.max() < (1 << (QB - 1))  # fits int8
        cbits = (code[w].astype(np.int64) >> (31 - j)) & 1
        assert int((q8 * cbits).sum()) == oracle.popcount_ip(planes, code)


def test_code_word_expansion_to_bytes():
    """The list scan's B operand: a code word (dim 32w + j -> bit 31 - j) becomes 32 bytes 0 / 1,
    byte j = dim 32w + j, by a bit reversal and, per nibble, a multiply by 0x00204081 masked with
    0x01010101 (the four shifted copies of the nibble do not overlap, so nothing carries)."""
    rng = np.random.default_rng(5)
    words = np.concatenate([rng.integers(0, 2 ** 32, 2000, dtype=np.uint64),
                            np.array([0, 0xFFFFFFFF, 0x80000001, 0x0F0F0F0F], np.uint64)])
    for c in words.tolist():
        r = int("{:032b}".format(c)[::-1], 2)  # __brev
        out = []
        for i in range(8):
            o = ((((r >> (4 * i)) & 0xF) * 0x00204081) & 0xFFFFFFFF) & 0x01010101
            out += [(o >> (8 * b)) & 0xFF for b in range(4)]  # little-endian bytes of the word
        assert out == [(c >> (31 - j)) & 1 for j in range(32)], hex(c)


# ------------------------------------------------------------------------------------------
# GPU
# ------------------------------------------------------------------------------------------
def _index(oracle, X, C, lab, bits=1):
    from neurosamble_b200 import IndexIVFRaBitQ
    idx = IndexIVFRaBitQ(X.shape[1], C.shape[0], seed=7, bits_per_dim=bits)
    idx.set_centroids(C)
    idx.add(X, labels=lab)
    oix = oracle.build(X, C, lab, idx.rotation(), idx.query_scale, bits_per_dim=bits,
                       tex=idx.info().ex_scale if bits > 1 else None)
    oix.t8 = oracle.query_scale(oix.dp, 7, 7)
    return idx, oix


@pytest.fixture(scope="module")
def gcase(oracle):
    X, Q = mixture(30000, 128, 60, 0.3, 400, seed=23)
    C, _ = oracle.kmeans(X[::5], 48, iters=4)
    lab = oracle.assign(X, C)
    idx, oix = _index(oracle, X, C, lab)
    return idx, oix, X, Q, C, lab


@pytest.mark.gpu
@pytest.mark.parametrize("bits,R,nprobe", [(4, 40, 8), (4, 100, 16), (8, 40, 8), (4, 10, 48)])
def test_list_scan_stage_bit_exact(oracle, gcase, bits, R, nprobe):
    """rbq_scan_lists against the oracle's list scan from the same thresholds: candidates,
    distances and the scanned / admitted counters."""
    import torch
    from neurosamble_b200 import _lib
    from neurosamble_b200.index import _ptr, _stream_ptr
    idx, oix, X, Q, C, lab = gcase
    Qr = oracle.rotate(Q, oix.P)
    nq = Qr.shape[0]
    pl, de, k1, _ = oracle.query_prep(Qr, oix.t4 if bits == 4 else oix.t8, bits)
    probes, g = oracle.coarse(Qr, oix.c_rot, nprobe)
    tau = oracle.bound_seed(oix, pl, de, k1, probes, g, R)
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a).view(dt)).cuda()
    qr, pld, ded, k1d = t(Qr, np.float32), t(pl, np.int32), t(de, np.float32), t(k1, np.float32)
    pd, gd, taud = t(probes, np.int32), t(g, np.float32), t(tau, np.float32)
    ids = torch.empty((nq, R), dtype=torch.int64, device="cuda")
    dist = torch.empty((nq, R), dtype=torch.float32, device="cuda")
    stats = torch.zeros(2, dtype=torch.int64, device="cuda")
    _lib.call("rbq_scan_lists", idx.handle, _ptr(qr), _ptr(pld), _ptr(ded), _ptr(k1d), nq, _ptr(pd), _ptr(gd),
              nprobe, 0, _ptr(taud), R, _ptr(ids), _ptr(dist), _ptr(stats), bits, _stream_ptr(idx.device))
    torch.cuda.synchronize()
    oi, od, ost = oracle.list_scan(oix, Qr, pl, de, k1, probes, g, R, tau, with_stats=True)
    assert np.array_equal(ids.cpu().numpy(), oi)
    assert np.array_equal(u32(dist.cpu().numpy()), u32(od))
    assert stats.cpu().tolist() == ost.tolist()


@pytest.mark.gpu
@pytest.mark.parametrize("bits,R", [(4, 0), (4, 40), (8, 40), (4, 200)])
def test_list_scan_search_bit_exact(oracle, gcase, bits, R):
    idx, oix, X, Q, C, lab = gcase
    idx.nprobe, idx.k_rerank, idx.query_bits, idx.scan_kind = 12, R, bits, 2
    try:
        for qs in (Q, Q[:3]):
            d, i = idx.search(qs, 10)
            d2, i2 = oracle.search(oix, qs, 10, 12, R, query_bits=bits, scan_kind=2)
            assert np.array_equal(i, i2) and np.array_equal(u32(d), u32(d2))
        # the fixed thresholds lose nothing against the tile scan's tightening ones
        _, gt = oracle.knn_exact(X, Q, 10)
        rec_list = oracle.recall(idx.search(Q, 10)[1], gt)
        idx.scan_kind = 1
        assert rec_list >= oracle.recall(idx.search(Q, 10)[1], gt) - 0.005
    finally:
        idx.query_bits, idx.scan_kind = 4, 0


@pytest.mark.gpu
def test_scan_kinds_match_the_oracle(oracle, gcase):
    """scan_kind 0 (auto: here the list scan for 400 queries x 12 probes over 48 lists, the tile
    scan for 5 queries), 1 and 2 each equal the oracle's search of that kind."""
    idx, oix, X, Q, C, lab = gcase
    idx.nprobe, idx.k_rerank = 12, 40
    try:
        for kind in (0, 1, 2):
            idx.scan_kind = kind
            for qs in (Q, Q[:5]):
                d, i = idx.search(qs, 10)
                d2, i2 = oracle.search(oix, qs, 10, 12, 40, scan_kind=kind)
                assert np.array_equal(i, i2) and np.array_equal(u32(d), u32(d2))
    finally:
        idx.scan_kind = 0


@pytest.mark.gpu
@pytest.mark.parametrize("d", [32, 96, 100, 256, 768])
def test_list_scan_other_dimensions(oracle, d):
    """Padded dims that fill part of a 128-byte chunk (32, 96), one or more chunks (128, 256) and
    six chunks (768)."""
    X, Q = mixture(6000, d, 20, 0.3, 120, seed=d)
    C, _ = oracle.kmeans(X[::3], 16, iters=3)
    lab = oracle.assign(X, C)
    idx, oix = _index(oracle, X, C, lab)
    idx.nprobe, idx.k_rerank, idx.scan_kind = 6, 30, 2
    d1, i1 = idx.search(Q, 10)
    d2, i2 = oracle.search(oix, Q, 10, 6, 30, scan_kind=2)
    assert np.array_equal(i1, i2) and np.array_equal(u32(d1), u32(d2))


@pytest.mark.gpu
def test_list_scan_extra_bits(oracle):
    X, Q = mixture(20000, 128, 40, 0.3, 300, seed=31)
    C, _ = oracle.kmeans(X[::4], 40, iters=3)
    lab = oracle.assign(X, C)
    idx, oix = _index(oracle, X, C, lab, bits=4)
    idx.nprobe, idx.k_rerank, idx.scan_kind = 8, 0, 2
    d1, i1 = idx.search(Q, 10)
    d2, i2 = oracle.search(oix, Q, 10, 8, 0, scan_kind=2)
    assert np.array_equal(i1, i2) and np.array_equal(u32(d1), u32(d2))


@pytest.mark.gpu
def test_overflowed_rows_take_the_fixed_threshold_tile_scan(oracle):
    """Uniform random vectors in 128 dims are nearly equidistant: the bound seed admits most of
    a query's 20,000 probed vectors, far past the 2,048-entry candidate row, so those queries are
    answered by the tile scan under the same fixed thresholds, with the same result."""
    import torch
    from neurosamble_b200 import _lib
    from neurosamble_b200.index import _ptr, _stream_ptr
    rng = np.random.default_rng(4)
    X = rng.standard_normal((20000, 128)).astype(np.float32)
    Q = rng.standard_normal((40, 128)).astype(np.float32)
    C, _ = oracle.kmeans(X[::4], 16, iters=3)
    lab = oracle.assign(X, C)
    idx, oix = _index(oracle, X, C, lab)
    idx.nprobe, idx.k_rerank, idx.scan_kind = 16, 10, 2
    d1, i1 = idx.search(Q, 10)
    d2, i2, st = oracle.search(oix, Q, 10, 16, 10, scan_kind=2, with_stats=True)
    assert st[1] > 2048 * 4  # several rows overflowed
    assert np.array_equal(i1, i2) and np.array_equal(u32(d1), u32(d2))
    # the stage's counters count every admitted vector once, overflowed rows included
    Qr = oracle.rotate(Q, oix.P)
    pl, de, k1, _ = oracle.query_prep(Qr, oix.t4, 4)
    probes, g = oracle.coarse(Qr, oix.c_rot, 16)
    tau = oracle.bound_seed(oix, pl, de, k1, probes, g, 10)
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a).view(dt)).cuda()
    ids = torch.empty((40, 10), dtype=torch.int64, device="cuda")
    dist = torch.empty((40, 10), dtype=torch.float32, device="cuda")
    stats = torch.zeros(2, dtype=torch.int64, device="cuda")
    # the device copies are held by name until the stage has run
    qr, pld, ded, k1d = t(Qr, np.float32), t(pl, np.int32), t(de, np.float32), t(k1, np.float32)
    pd, gd, taud = t(probes, np.int32), t(g, np.float32), t(tau, np.float32)
    _lib.call("rbq_scan_lists", idx.handle, _ptr(qr), _ptr(pld), _ptr(ded), _ptr(k1d), 40, _ptr(pd), _ptr(gd), 16, 0,
              _ptr(taud), 10, _ptr(ids), _ptr(dist), _ptr(stats), 4, _stream_ptr(idx.device))
    torch.cuda.synchronize()
    oi, od, ost = oracle.list_scan(oix, Qr, pl, de, k1, probes, g, 10, tau, with_stats=True)
    assert np.array_equal(ids.cpu().numpy(), oi) and np.array_equal(u32(dist.cpu().numpy()), u32(od))
    assert stats.cpu().tolist() == ost.tolist()


@pytest.mark.gpu
@pytest.mark.parametrize("K,R", [(64, 200), (16, 40)])
def test_list_scan_seed_from_leading_lists_or_the_nearest(oracle, K, R):
    """Lists smaller than R (6,000 vectors in 64 lists, R 200) need the separate bound-seed launch
    over the leading lists; lists of R or more (16 lists, R 40) let the nearest probe's tile scan
    seed itself.  Both equal the oracle's list search."""
    X, Q = mixture(6000, 64, 30, 0.3, 150, seed=K)
    C, _ = oracle.kmeans(X[::3], K, iters=3)
    lab = oracle.assign(X, C)
    idx, oix = _index(oracle, X, C, lab)
    idx.nprobe, idx.k_rerank, idx.scan_kind = 8, R, 2
    d1, i1 = idx.search(Q, 10)
    d2, i2 = oracle.search(oix, Q, 10, 8, R, scan_kind=2)
    assert np.array_equal(i1, i2) and np.array_equal(u32(d1), u32(d2))
    sizes = np.diff(oix.list_off)
    assert (sizes.min() < R) == (K == 64)
