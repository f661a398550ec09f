"""rbq_scan_noalloc: the list scan for callers that cannot allocate GPU memory at search time.

Such a caller (for example a server whose device memory is all handed out up front by its
own pool, or a latency-critical search thread that must not trigger an allocation) gets the
same candidates as rbq_scan while the library uses only its fixed, compiled-in scratch array.
These tests call both entry points through the C ABI on the same inputs and require equal
results on two calls in a row (the array keeps the previous call's contents, so the second
call also shows that nothing stale leaks through), and check that a batch too large for the
array is refused before any work is queued.  This file sorts last so that a run stopping at
the first failure has run every other test already; it builds its own index, so it also
passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from conftest import mixture

SCRATCH_BYTES = 32 << 20  # RBQ_NOALLOC_SCRATCH_BYTES in include/rbq.h


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _round256(v):
    return (v + 255) // 256 * 256


def test_size_rule_rejects_before_touching_the_index():
    """Host-side check (no GPU needed): an oversized request fails with RBQ_ERR_INVALID and a
    message naming the limit; the index pointer is not used."""
    from neurosamble_b200 import _lib
    L = _lib.lib()
    dummy = ctypes.c_void_p(1)  # never dereferenced: the size rule is checked first
    buf = ctypes.c_void_p(1)
    nq, R = 9000, 512  # 9000 * 512 * 8 bytes > 32 MiB
    st = L.rbq_scan_noalloc(dummy, buf, buf, buf, buf, nq, buf, buf, 8, 0, None, R, 1, 1, 0, buf, buf, None,
                            4, None)
    assert st == 1
    msg = L.rbq_last_error().decode()
    assert "static scratch holds 33554432 bytes" in msg


def _stage(idx, Q, nprobe):
    import torch
    from neurosamble_b200 import _lib
    from neurosamble_b200.index import _stream_ptr
    nq, dp = Q.shape[0], idx.info().padded_dim
    s = _stream_ptr(idx.device)
    q = torch.from_numpy(Q).cuda()
    qr = torch.empty((nq, dp), dtype=torch.float32, device="cuda")
    planes = torch.empty((nq, 4, dp // 32), dtype=torch.int32, device="cuda")
    delta = torch.empty(nq, dtype=torch.float32, device="cuda")
    k1 = torch.empty(nq, dtype=torch.float32, device="cuda")
    probes = torch.empty((nq, nprobe), dtype=torch.int32, device="cuda")
    g = torch.empty((nq, nprobe), dtype=torch.float32, device="cuda")
    _lib.call("rbq_rotate", idx.handle, _p(q), nq, _p(qr), s)
    _lib.call("rbq_coarse", idx.handle, _p(qr), nq, nprobe, 0, _p(probes), _p(g), s)
    _lib.call("rbq_query_prep", idx.handle, _p(qr), nq, _p(planes), _p(delta), _p(k1), 4, s)
    return qr, planes, delta, k1, probes, g


def _run(idx, name, st, nprobe, R, prune, slices):
    import torch
    from neurosamble_b200 import _lib
    from neurosamble_b200.index import _stream_ptr
    qr, planes, delta, k1, probes, g = st
    nq = qr.shape[0]
    ids = torch.full((nq, R), -7, dtype=torch.int64, device="cuda")
    dist = torch.full((nq, R), -7.0, dtype=torch.float32, device="cuda")
    stats = torch.zeros(2, dtype=torch.int64, device="cuda")
    init = (None, None) if name == "rbq_scan" else ()  # rbq_scan's initial candidates: none
    _lib.call(name, idx.handle, _p(qr), _p(planes), _p(delta), _p(k1), nq, _p(probes), _p(g), nprobe, 0, None, *init, R,
              prune, slices, 0, _p(ids), _p(dist), _p(stats), 4, _stream_ptr(idx.device))
    torch.cuda.synchronize()
    return ids.cpu().numpy(), dist.cpu().numpy(), stats.cpu().numpy()


@pytest.mark.gpu
def test_noalloc_scan_matches_scan_on_two_calls_in_a_row():
    from neurosamble_b200 import IndexIVFRaBitQ, _lib
    X, Q = mixture(20000, 128, 40, 0.3, 400, seed=21)
    idx = IndexIVFRaBitQ(128, 64, seed=7, kmeans_iters=5)
    idx.train(X)
    idx.add(X)
    calls = [(Q[:300], 8, 40, 1, 1), (Q[300:337], 16, 100, 0, 4)]
    for Qc, nprobe, R, prune, slices in calls:
        assert _round256(len(Qc) * slices * R * 8) + (_round256(len(Qc) * R * 8) if slices > 1 else 0) <= SCRATCH_BYTES
        st = _stage(idx, Qc, nprobe)
        ref = _run(idx, "rbq_scan", st, nprobe, R, prune, slices)
        # arm the library's allocation-failure injection: the very next device allocation it
        # makes would fail with RBQ_ERR_OOM, so a successful call proves that it made none
        L = _lib.lib()
        assert L.rbq_debug_fail_alloc(0) == 0
        try:
            got = _run(idx, "rbq_scan_noalloc", st, nprobe, R, prune, slices)
        finally:
            L.rbq_debug_fail_alloc(-1)
        assert np.array_equal(got[0], ref[0])
        assert np.array_equal(got[1].view(np.uint32), ref[1].view(np.uint32))  # the tests' tolerance: bit-exact
        assert np.array_equal(got[2], ref[2])
        assert (got[0] >= 0).any()


@pytest.mark.gpu
def test_noalloc_scan_refuses_batches_beyond_the_scratch():
    import torch
    from neurosamble_b200 import IndexIVFRaBitQ, _lib
    from neurosamble_b200.index import _stream_ptr
    X, Q = mixture(4000, 64, 8, 0.3, 10, seed=3)
    idx = IndexIVFRaBitQ(64, 16, seed=7, kmeans_iters=3)
    idx.train(X)
    idx.add(X)
    nq, R, nprobe = 1100, 4096, 4  # 1100 * 4096 * 8 bytes > 32 MiB; every input is real and in bounds
    qr = torch.zeros((nq, 64), dtype=torch.float32, device="cuda")
    planes = torch.zeros((nq, 4, 2), dtype=torch.int32, device="cuda")
    delta = torch.zeros(nq, dtype=torch.float32, device="cuda")
    k1 = torch.zeros(nq, dtype=torch.float32, device="cuda")
    probes = torch.zeros((nq, nprobe), dtype=torch.int32, device="cuda")
    g = torch.ones((nq, nprobe), dtype=torch.float32, device="cuda")
    ids = torch.empty((nq, R), dtype=torch.int64, device="cuda")
    dist = torch.empty((nq, R), dtype=torch.float32, device="cuda")
    st = _lib.lib().rbq_scan_noalloc(idx.handle, _p(qr), _p(planes), _p(delta), _p(k1), nq, _p(probes), _p(g),
                                     nprobe, 0, None, R, 1, 1, 0, _p(ids), _p(dist), None, 4,
                                     _stream_ptr(idx.device))
    assert st == 1 and b"static scratch" in _lib.lib().rbq_last_error()
