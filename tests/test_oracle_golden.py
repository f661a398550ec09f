"""Pin the CPU oracle: published Philox vectors, hand-computed closed forms and the
independent pure-Python restatement in tests/golden/golden_small.npz."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "golden_small.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLDEN)


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


# Random123 known-answer vectors for philox4x32-10 (counter, key, output).
PHILOX_KAT = [
    ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
    ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
    ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
     (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
]


@pytest.mark.parametrize("ctr,key,expect", PHILOX_KAT)
def test_philox_known_answers(oracle, ctr, key, expect):
    assert oracle.philox(key, ctr).tolist() == list(expect)


def test_gaussian_stream_is_standard_normal(oracle):
    g = oracle.gaussian(123, 1, 0, 200000)
    assert abs(g.mean()) < 0.01 and abs(g.std() - 1.0) < 0.01
    assert np.array_equal(g[1000:1010], oracle.gaussian(123, 1, 1000, 10))


@pytest.mark.parametrize("dp", [32, 64, 128, 256])
def test_rotation_is_orthogonal_and_seeded(oracle, dp):
    P = oracle.make_rotation(dp, 7)
    assert np.abs(P.astype(np.float64) @ P.T.astype(np.float64) - np.eye(dp)).max() < 1e-5
    assert np.array_equal(bits(P), bits(oracle.make_rotation(dp, 7)))
    assert not np.array_equal(P, oracle.make_rotation(dp, 8))


def test_best_rescale_hand_case(oracle):
    # dim 2, o = (0.6, 0.8), ex_bits 1: t_end = 11/0.8, start levels (1, 1); the first
    # critical point t = 2/0.8 = 2.5 raises coordinate 1 and maximises <o_bar,o>/|o_bar|.
    assert oracle.best_rescale(np.array([0.6, 0.8]), 1) == pytest.approx(2.5, abs=1e-12)


def test_query_scale_is_deterministic(oracle):
    t = oracle.query_scale(128, 7)
    assert 20.0 < t < 80.0
    assert t == oracle.query_scale(128, 7)


@pytest.mark.parametrize("case", ["A", "B"])
def test_quantize_closed_form(oracle, gold, case):
    code, f3 = oracle.quantize_one(gold[case + "_y"], gold[case + "_c"])
    assert code.tolist() == gold[case + "_code"].tolist()
    assert np.array_equal(bits(f3), bits(gold[case + "_f3"]))


def test_query_prep_closed_form(oracle, gold):
    planes, delta, k1, codes = oracle.query_prep(gold["Q_q"][None, :], float(gold["Q_t4"][0]))
    assert codes[0, 0] == 7 and not codes[0, 1:].any()
    assert np.array_equal(planes[0], gold["Q_planes"])
    assert np.array_equal(bits(delta), bits(gold["Q_delta"]))
    assert np.array_equal(bits(k1), bits(gold["Q_k1"]))
    assert oracle.popcount_ip(planes[0], gold["A_code"]) == int(gold["AQ_acc"][0])


@pytest.mark.parametrize("dp", [64, 96])
def test_restated_random_cases(oracle, gold, dp):
    p = f"R{dp}_"
    Y, C, Qr = gold[p + "Y"], gold[p + "C"], gold[p + "Qr"]
    for i in range(Y.shape[0]):
        code, f3 = oracle.quantize_one(Y[i], C[i])
        assert np.array_equal(code, gold[p + "codes"][i])
        assert np.array_equal(bits(f3), bits(gold[p + "f3"][i]))
    planes, delta, k1, qcodes = oracle.query_prep(Qr, float(gold[p + "t4"][0]))
    assert np.array_equal(planes, gold[p + "planes"])
    assert np.array_equal(qcodes, gold[p + "qcodes"])
    assert np.array_equal(bits(delta), bits(gold[p + "delta"]))
    assert np.array_equal(bits(k1), bits(gold[p + "k1"]))
    G = gold[p + "G"]
    for q in range(Qr.shape[0]):
        for i in range(Y.shape[0]):
            acc = oracle.popcount_ip(planes[q], gold[p + "codes"][i])
            assert acc == int(gold[p + "acc"][q, i])
            est, low = oracle.estimate(gold[p + "f3"][i], G[q, i], acc, delta[q], k1[q])
            assert bits(np.float32(est)) == bits(gold[p + "est"][q, i])
            assert bits(np.float32(low)) == bits(gold[p + "low"][q, i])
            eip = oracle.exact_ip(Qr[q], gold[p + "codes"][i])
            assert bits(np.float32(eip)) == bits(gold[p + "eip"][q, i])


def test_popcount_equals_signed_code_dot_bits(oracle):
    """The plane popcount equals sum_d code_d * bit_d with codes in [-8, 7]."""
    rng = np.random.default_rng(5)
    dp = 128
    for _ in range(20):
        qc = rng.integers(-8, 8, dp)
        bitsv = rng.integers(0, 2, dp)
        planes = np.zeros((4, dp // 32), np.uint32)
        code = np.zeros(dp // 32, np.uint32)
        for j in range(dp):
            u = int(qc[j]) & 0xF
            for b in range(4):
                if (u >> b) & 1:
                    planes[b, j >> 5] |= np.uint32(1 << (31 - (j & 31)))
            if bitsv[j]:
                code[j >> 5] |= np.uint32(1 << (31 - (j & 31)))
        assert oracle.popcount_ip(planes, code) == int((qc * bitsv).sum())


def test_l2_exact_matches_float64(oracle):
    rng = np.random.default_rng(3)
    for d in (1, 31, 128, 300):
        x = rng.standard_normal(d).astype(np.float32)
        q = rng.standard_normal(d).astype(np.float32)
        ref = float(((x.astype(np.float64) - q.astype(np.float64)) ** 2).sum())
        assert oracle.l2_exact(x, q) == pytest.approx(ref, rel=1e-6)
