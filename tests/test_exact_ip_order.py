"""The exact 1-bit inner product's addition order, emulated in float32 on the CPU: the one-vector
form (32 lanes, byte j on lane j % 32, then an xor butterfly 16, 8, 4, 2, 1) and the four-vector
form (8-lane groups: lane k forms what lanes k, k + 8, k + 16, k + 24 hold, adds them in the
butterfly's first two levels, then xor 4, 2, 1 inside the group) give the same bits in every
lane.  The GPU kernels (warp_exact_ip, group8_exact_ip in rbq_search.cu) follow these orders."""
import numpy as np
import pytest

f32 = np.float32


def _bsum(u8, qb):
    """Sum of q over the set bits of one code byte, bit 7 first, from +0 (the kernels' order)."""
    b = f32(0.0)
    for jj in range(8):
        if (u8 >> (7 - jj)) & 1:
            b = f32(b + qb[jj])
    return b


def _leaf(code, q, lane, NB):
    """What lane `lane` of the one-vector form holds before the butterfly."""
    v = f32(0.0)
    for j in range(lane, NB, 32):
        v = f32(v + _bsum(code[j], q[8 * j:8 * j + 8]))
    return v


def warp_form(code, q, NB):
    v = [_leaf(code, q, l, NB) for l in range(32)]
    for off in (16, 8, 4, 2, 1):
        v = [f32(v[l] + v[l ^ off]) for l in range(32)]
    return v


def group_form(code, q, NB):
    t = []
    for k in range(8):
        v = [_leaf(code, q, k + 8 * h, NB) for h in range(4)]
        t.append(f32(f32(v[0] + v[2]) + f32(v[1] + v[3])))
    for off in (4, 2, 1):
        t = [f32(t[k] + t[k ^ off]) for k in range(8)]
    return t


@pytest.mark.parametrize("W", [1, 2, 3, 4, 6, 8, 12, 24])
def test_group_form_equals_warp_form_bit_for_bit(W):
    NB = 4 * W
    rng = np.random.default_rng(W)
    for trial in range(40):
        q = rng.standard_normal(8 * NB).astype(np.float32) * f32(10.0 ** rng.integers(-3, 3))
        code = rng.integers(0, 256, NB)
        if trial == 0:
            code[:] = 0      # no bit set: +0 everywhere
        elif trial == 1:
            code[:] = 255    # every bit set
        w = warp_form(code, q, NB)
        g = group_form(code, q, NB)
        assert len({x.tobytes() for x in w}) == 1  # every lane of the warp holds the same value
        assert len({x.tobytes() for x in g}) == 1  # every lane of the group holds the same value
        assert w[0].tobytes() == g[0].tobytes(), (W, trial, w[0], g[0])
