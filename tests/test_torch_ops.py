"""torch.ops.rbq.*: registration and shapes on CPU; on the GPU, every operator agrees bit for
bit with the C-ABI search it wraps."""
import numpy as np
import pytest
import torch

from conftest import mixture

OPS = ["search", "rotate", "query_prep", "coarse", "scan", "bound_seed", "rerank", "merge_results"]


def u32(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_ops_registered_with_shapes():
    import neurosamble_b200  # noqa: F401  (registers the operators)
    ops = torch.ops.rbq
    for name in OPS:
        assert hasattr(ops, name), name

    def m(*s, dt=torch.float32):
        return torch.empty(*s, dtype=dt, device="meta")

    assert ops.rotate(1, m(5, 100)).shape == (5, 128)
    planes, delta, k1 = ops.query_prep(1, m(5, 128))
    assert planes.shape == (5, 4, 4) and planes.dtype == torch.int32 and delta.shape == k1.shape == (5,)
    probes, g = ops.coarse(1, m(5, 128), 7, 0)
    assert probes.shape == g.shape == (5, 7) and probes.dtype == torch.int32
    ids, dist = ops.scan(1, m(5, 128), planes, delta, k1, probes, g, 40, True, 1, 0, None)
    assert ids.shape == dist.shape == (5, 40) and ids.dtype == torch.int64
    assert ops.bound_seed(1, m(5, 128), planes, delta, k1, probes, g, 40, 0).shape == (5,)
    d, i = ops.rerank(1, m(5, 100), m(5, 40, dt=torch.int64), 10)
    assert d.shape == i.shape == (5, 10) and i.dtype == torch.int64
    d, i = ops.merge_results(m(3, 5, 10), m(3, 5, 10, dt=torch.int64))
    assert d.shape == i.shape == (5, 10)
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        d, i = ops.search(1, torch.empty(6, 64, device="cuda"), 4, 3, 0, True, 0, -1)
        assert d.shape == (6, 4) and i.dtype == torch.int64 and d.device.type == "cuda"


def test_ops_reject_host_tensors_before_any_library_call():
    import neurosamble_b200  # noqa: F401
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        torch.ops.rbq.rotate(1, torch.zeros(3, 32))
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        torch.ops.rbq.merge_results(torch.zeros(2, 3, 4), torch.zeros(2, 3, 4, dtype=torch.int64))


@pytest.fixture(scope="module")
def built():
    from neurosamble_b200 import IndexIVFRaBitQ
    X, Q = mixture(20000, 96, 60, 0.3, 700, seed=21)
    idx = IndexIVFRaBitQ(96, 64, seed=3, kmeans_iters=4)
    idx.train(X)
    idx.add(X)
    return idx, X, Q


@pytest.mark.gpu
def test_search_op_equals_index_search(built):
    idx, X, Q = built
    idx.nprobe, idx.k_rerank = 8, 40
    q = torch.from_numpy(Q).cuda()
    d1, i1 = idx.search(q, 10)
    d2, i2 = torch.ops.rbq.search(idx.handle.value, q, 10, 8, 40, True, 0, -1)
    torch.cuda.synchronize()
    assert torch.equal(i1, i2) and np.array_equal(u32(d1.cpu().numpy()), u32(d2.cpu().numpy()))


@pytest.mark.gpu
def test_stage_ops_compose_to_the_search(built):
    """rotate -> coarse -> query_prep -> scan -> rerank (one slice, no seed launch) is the
    search of a 700-query batch (probe_split 1, seeded 0)."""
    idx, X, Q = built
    h, P, R, k = idx.handle.value, 8, 40, 10
    q = torch.from_numpy(Q).cuda()
    ops = torch.ops.rbq
    qr = ops.rotate(h, q)
    probes, g = ops.coarse(h, qr, P, 0)
    planes, delta, k1 = ops.query_prep(h, qr)
    cand_ids, cand_dist = ops.scan(h, qr, planes, delta, k1, probes, g, R, True, 1, 0, None)
    d, i = ops.rerank(h, q, cand_ids, k)
    d2, i2 = ops.search(h, q, k, P, R, True, 1, 0)
    torch.cuda.synchronize()
    assert torch.equal(i, i2) and np.array_equal(u32(d.cpu().numpy()), u32(d2.cpu().numpy()))
    # candidates are ascending by estimate and every returned id is one of them
    cd = cand_dist.cpu().numpy()
    assert np.all(np.diff(cd, axis=1)[np.isfinite(cd[:, 1:])] >= 0)
    ci = cand_ids.cpu().numpy()
    for a, b in zip(i.cpu().numpy()[:50], ci[:50]):
        assert set(a[a >= 0].tolist()) <= set(b[b >= 0].tolist())
    # the seeded search (seeded = 1) is bound_seed over the nearest probe, then the scan of all
    # probes from that threshold
    tau = ops.bound_seed(h, qr, planes, delta, k1, probes[:, :1].contiguous(), g[:, :1].contiguous(), R, 0)
    ids_s, _ = ops.scan(h, qr, planes, delta, k1, probes, g, R, True, 1, 0, tau)
    d3, i3 = ops.rerank(h, q, ids_s, k)
    d4, i4 = ops.search(h, q, k, P, R, True, 1, 1)
    torch.cuda.synchronize()
    assert torch.equal(i3, i4) and np.array_equal(u32(d3.cpu().numpy()), u32(d4.cpu().numpy()))


@pytest.mark.gpu
def test_merge_results_op_reassembles_a_split_result(built):
    idx, X, Q = built
    q = torch.from_numpy(Q[:300]).cuda()
    d, i = torch.ops.rbq.search(idx.handle.value, q, 10, 8, 40, True, 0, -1)
    inf = torch.full_like(d[:, :5], float("inf"))
    neg = torch.full_like(i[:, :5], -1)
    parts_d = torch.stack([torch.cat([d[:, 0::2], inf], 1), torch.cat([d[:, 1::2], inf], 1)])
    parts_i = torch.stack([torch.cat([i[:, 0::2], neg], 1), torch.cat([i[:, 1::2], neg], 1)])
    md, mi = torch.ops.rbq.merge_results(parts_d, parts_i)
    torch.cuda.synchronize()
    assert torch.equal(mi, i) and torch.equal(md, d)
