"""Generate tests/golden/golden_small.npz: known-answer vectors for the 1-bit RaBitQ path.

Independent of the C++ oracle: a pure-Python (numpy float32 scalar) restatement of the
reference formulas, run on small cases only, plus closed-form cases computed by hand.

Formulas restated (reference paths relative to third-party/cuvs_rabitq/cpp/src/neighbors/
ivf_rabitq/gpu_index/):
  * quantizer_gpu.cu:109-172, 251-338  codes (dim 32w+j -> bit 31-j), f_add, f_rescale, f_err
  * searcher_gpu_quantize_query.cu:655-793  4-bit query codes, delta, bit planes
  * searcher_gpu_quantize_query.cu:233-281  popcount inner product and the estimator
  * ivf_gpu.cu:1451-1490  k1 = -0.5 * sum(q)
Reductions follow this project's fixed order: double sums in dimension order, rounded to
float32 once.

Run: python tests/golden/make_golden.py   (rewrites the .npz next to this file)
"""
from __future__ import annotations

import os

import numpy as np

F = np.float32
HERE = os.path.dirname(os.path.abspath(__file__))


def quantize_one(y, c):
    dp = len(y)
    r = [F(y[j]) - F(c[j]) for j in range(dp)]
    l2d = 0.0
    for v in r:
        l2d += float(v) * float(v)
    l2 = F(l2d)
    norm = F(np.sqrt(l2))  # float32 sqrt: correctly rounded, like sqrtf
    ipr = 0.0
    ipc = 0.0
    words = [0] * (dp // 32)
    for j in range(dp):
        bit = 1 if (norm > F(0) and r[j] > F(0)) else 0
        if bit:
            words[j >> 5] |= 1 << (31 - (j & 31))
        xu = 0.5 if bit else -0.5
        ipr += float(r[j]) * xu
        ipc += float(F(c[j])) * xu
    ip_resi = F(ipr)
    ip_cent = F(ipc)
    xu_sq = F(0.25) * F(dp)
    if ip_resi == F(0):
        ip_resi = F(np.inf)
    l2_norm = F(np.sqrt(np.maximum(l2, F(0))))
    denom = ip_resi
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        fadd = l2 + (F(2) * l2) * (ip_cent / denom)
        fres = (F(-2) * l2) / denom
        ratio = (l2 * xu_sq) / (denom * denom)
        inner = (ratio - F(1)) / np.maximum(F(dp - 1), F(1))
        inner = np.maximum(inner, F(0))
        ferr = F(2) * ((l2_norm * F(1.9)) * F(np.sqrt(inner)))
    return np.array(words, np.uint32), np.array([fadd, fres, ferr], np.float32)


def query_prep(q, t4):
    dp = len(q)
    s2 = 0.0
    s1 = 0.0
    for v in q:
        s2 += float(v) * float(v)
        s1 += float(v)
    norm = F(np.sqrt(F(s2)))
    norm_inv = F(1) / norm if norm > F(0) else F(0)
    codes = []
    ipd = 0.0
    xs = 0
    for j in range(dp):
        val = F(q[j]) * norm_inv
        tv = F(t4) * val
        cv = int(np.rint(tv))  # round half to even
        cv = max(-8, min(7, cv))
        codes.append(cv)
        ipd += float(q[j]) * float(cv)
        xs += cv * cv
    ip = F(ipd)
    xu_sq = F(xs)
    nq_ = F(np.sqrt(np.maximum(xu_sq, F(0))))
    if norm > F(1e-6) and nq_ > F(1e-6):
        cosv = ip / (norm * nq_)
        delta = (norm / nq_) * cosv
    else:
        delta = F(0)
    k1 = F(s1) * F(-0.5)
    w = dp // 32
    planes = np.zeros((4, w), np.uint32)
    for j, cv in enumerate(codes):
        u = cv & 0xF
        for b in range(4):
            if (u >> b) & 1:
                planes[b, j >> 5] |= np.uint32(1 << (31 - (j & 31)))
    return planes, F(delta), F(k1), np.array(codes, np.int8)


def popcount_ip(planes, code):
    acc = 0
    for w in range(len(code)):
        c = int(code[w])
        for b in range(3):
            acc += bin(int(planes[b, w]) & c).count("1") << b
        acc -= bin(int(planes[3, w]) & c).count("1") << 3
    return acc


def byte_sum(q, code, j):
    """Sum of q over the set bits of byte j of the MSB-first bit stream (dims 8j..8j+7)."""
    byte = (int(code[j >> 2]) >> (24 - 8 * (j & 3))) & 0xFF
    s = F(0)
    for jj in range(8):
        if (byte >> (7 - jj)) & 1:
            s = s + F(q[8 * j + jj])
    return s


def exact_ip(q, code):
    """32 lane sums (lane l: bytes l, l+32, ... in order), then an xor butterfly 16..1."""
    nb = 4 * len(code)
    v = []
    for lane in range(32):
        s = F(0)
        for j in range(lane, nb, 32):
            s = s + byte_sum(q, code, j)
        v.append(s)
    for off in (16, 8, 4, 2, 1):
        v = [v[lane] + v[lane ^ off] for lane in range(32)]
    return F(v[0])


def estimate(f3, g, acc, delta, k1):
    base = f3[0] + F(g)
    ip = F(acc) * F(delta)
    est = base + f3[1] * (ip + F(k1))
    low = est - f3[2] * F(np.sqrt(F(g)))
    return F(est), F(low)


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    # Closed-form case A: c = 0, r = +-0.5 alternating (D = 32).
    yA = np.array([0.5 if j % 2 == 0 else -0.5 for j in range(32)], np.float32)
    cA = np.zeros(32, np.float32)
    out["A_y"], out["A_c"] = yA, cA
    out["A_code"] = np.array([0xAAAAAAAA], np.uint32)
    out["A_f3"] = np.array([8.0, -2.0, 0.0], np.float32)
    # Closed-form case B: c_j = 1 on even dims, same residual: ip_cent = 8 -> f_add = 24.
    cB = np.array([1.0 if j % 2 == 0 else 0.0 for j in range(32)], np.float32)
    out["B_y"], out["B_c"] = cB + yA, cB
    out["B_code"] = np.array([0xAAAAAAAA], np.uint32)
    out["B_f3"] = np.array([24.0, -2.0, 0.0], np.float32)
    # Closed-form case Q: one-hot query e_0 with t4 = 23.25 -> code_0 = 7, delta = 1/7, k1 = -0.5.
    qQ = np.zeros(32, np.float32)
    qQ[0] = 1.0
    out["Q_q"] = qQ
    out["Q_t4"] = np.array([23.25], np.float32)
    pl = np.zeros((4, 1), np.uint32)
    pl[0, 0] = pl[1, 0] = pl[2, 0] = 0x80000000
    out["Q_planes"] = pl
    out["Q_delta"] = np.array([(F(1) / F(7)) * (F(7) / (F(1) * F(7)))], np.float32)
    out["Q_k1"] = np.array([-0.5], np.float32)
    # Popcount of code 0xAAAAAAAA (dim 0 set) against code 7 on dim 0 -> 7.
    out["AQ_acc"] = np.array([7], np.int32)
    # Restated random cases, D = 64 and D = 96.
    for dp in (64, 96):
        n, nq = 24, 6
        Y = rng.standard_normal((n, dp)).astype(np.float32)
        C = (0.3 * rng.standard_normal((n, dp))).astype(np.float32)
        Qr = rng.standard_normal((nq, dp)).astype(np.float32)
        t4 = F(38.5)
        G = (np.abs(rng.standard_normal((nq, n))) + 0.1).astype(np.float32)
        codes = np.zeros((n, dp // 32), np.uint32)
        f3 = np.zeros((n, 3), np.float32)
        for i in range(n):
            codes[i], f3[i] = quantize_one(Y[i], C[i])
        planes = np.zeros((nq, 4, dp // 32), np.uint32)
        delta = np.zeros(nq, np.float32)
        k1 = np.zeros(nq, np.float32)
        qcodes = np.zeros((nq, dp), np.int8)
        for q in range(nq):
            planes[q], delta[q], k1[q], qcodes[q] = query_prep(Qr[q], t4)
        acc = np.zeros((nq, n), np.int32)
        est = np.zeros((nq, n), np.float32)
        low = np.zeros((nq, n), np.float32)
        eip = np.zeros((nq, n), np.float32)
        for q in range(nq):
            for i in range(n):
                acc[q, i] = popcount_ip(planes[q], codes[i])
                est[q, i], low[q, i] = estimate(f3[i], G[q, i], acc[q, i], delta[q], k1[q])
                eip[q, i] = exact_ip(Qr[q], codes[i])
        p = f"R{dp}_"
        out.update({p + "Y": Y, p + "C": C, p + "Qr": Qr, p + "t4": np.array([t4], np.float32), p + "G": G,
                    p + "codes": codes, p + "f3": f3, p + "planes": planes, p + "delta": delta, p + "k1": k1,
                    p + "qcodes": qcodes, p + "acc": acc, p + "est": est, p + "low": low, p + "eip": eip})
    np.savez_compressed(os.path.join(HERE, "golden_small.npz"), **out)
    print("wrote", os.path.join(HERE, "golden_small.npz"), len(out), "arrays")


if __name__ == "__main__":
    main()
