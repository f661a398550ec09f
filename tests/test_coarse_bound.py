"""The coarse quantiser's shortlist proof rests on a bound E on |tf32 score - exact score|, score =
|c|^2 - 2 <q, c> (tf32_score_bound in rbq_search.cu: (2^-7 + d 2^-21) |q| |c|max + 2^-19 (|q|^2 +
|c|max^2)).  Emulated here on the CPU with the worst operand conversion (truncation of each fp32
operand to tf32's 10 mantissa bits) and fp32 accumulation of the exact tf32 products in several
orders, the error stays within half of E for random and adversarial vectors."""
import numpy as np
import pytest

f32 = np.float32


def tf32_trunc(x):
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


def bound(qn2, cmax2, d):
    rel = f32(0.0078125) + f32(d) * f32(4.76837158e-7)
    return rel * np.sqrt(f32(qn2 * cmax2)) + f32(1.90734863e-6) * f32(qn2 + cmax2)


def scores(q, C, order, rng):
    """tf32 scores of q against the rows of C: products exact in fp32 (11 x 11 mantissa bits),
    summed in fp32 sequentially in the given order, then cn - 2 ip in fp32."""
    prod = tf32_trunc(q)[None, :] * tf32_trunc(C)  # exact
    if order == "reverse":
        prod = prod[:, ::-1]
    elif order == "shuffled":
        prod = prod[:, rng.permutation(prod.shape[1])]
    if order == "pairwise":
        ip = prod.sum(axis=1, dtype=np.float32)
    else:
        ip = np.cumsum(prod, axis=1, dtype=np.float32)[:, -1]
    cn = (C.astype(np.float64) ** 2).sum(1).astype(np.float32)
    return (cn - f32(2.0) * ip).astype(np.float32)


@pytest.mark.parametrize("d", [32, 128, 256, 768])
@pytest.mark.parametrize("kind", ["gauss", "normalised", "large", "cancel"])
def test_tf32_score_error_within_half_the_bound(d, kind):
    rng = np.random.default_rng(d + len(kind))
    C = rng.standard_normal((400, d)).astype(np.float32)
    q = rng.standard_normal(d).astype(np.float32)
    if kind == "normalised":
        C /= np.linalg.norm(C, axis=1, keepdims=True)
        q /= np.linalg.norm(q)
    elif kind == "large":
        C *= f32(1e3)
        q *= f32(1e-2)
    elif kind == "cancel":  # rows nearly orthogonal to q with large entries that cancel
        C -= np.outer(C @ q / (q @ q), q).astype(np.float32)
        C *= f32(50.0)
    exact = (C.astype(np.float64) ** 2).sum(1) - 2.0 * (C.astype(np.float64) @ q.astype(np.float64))
    qn2 = f32((q.astype(np.float64) ** 2).sum())
    cmax2 = f32((C.astype(np.float64) ** 2).sum(1).max())
    E = float(bound(qn2, cmax2, d))
    for order in ("sequential", "reverse", "shuffled", "pairwise"):
        err = np.abs(scores(q, C, order, rng).astype(np.float64) - exact).max()
        assert err <= 0.5 * E, (d, kind, order, err, E)
