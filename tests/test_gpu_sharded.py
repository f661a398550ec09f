"""List-sharded search on 2 GPUs (NCCL): the merged result of ShardedIndexIVFRaBitQ (split
front end, seeded threshold shared by an all-reduce, one all-gather of the results) equals the
oracle's sharded search (exchange=True) merged by (distance, id), bit for bit.  Skipped with
fewer than 2 GPUs."""
import os
import pickle
import socket
import tempfile
from datetime import timedelta

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ngpu():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, outdir):
    import torch
    import torch.distributed as dist

    from conftest import mixture
    from oracle import oracle as O
    from neurosamble_b200.sharded import ShardedIndexIVFRaBitQ

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    X, Q = mixture(20000, 128, 40, 0.3, 200, seed=31)
    C, _ = O.kmeans(X[::4], 64, iters=4)
    lab = O.assign(X, C)
    idx = ShardedIndexIVFRaBitQ(128, 64, seed=7, device=rank)
    idx.local.set_centroids(C)
    idx.add(X, labels=lab)
    idx.nprobe, idx.k_rerank, idx.probe_split = 12, 40, 1
    st = torch.zeros(2, dtype=torch.int64, device=f"cuda:{rank}")
    d, i = idx.search(Q, 10, stats=st)
    stats = [torch.zeros(2, dtype=torch.int64, device=f"cuda:{rank}") for _ in range(world)]
    dist.all_gather(stats, st)
    # the list scan (scan_kind 2): seeds and the nearest list's threshold all-reduced
    idx.scan_kind = 2
    stl = torch.zeros(2, dtype=torch.int64, device=f"cuda:{rank}")
    dl, il = idx.search(Q, 10, stats=stl)
    idx.scan_kind = 0
    stats_l = [torch.zeros(2, dtype=torch.int64, device=f"cuda:{rank}") for _ in range(world)]
    dist.all_gather(stats_l, stl)
    # build(): with the given centroids and labels, and by training (rank 0 trains, the table is
    # broadcast), against train() + add() on the same rows; a second build is refused
    same = []
    b1 = ShardedIndexIVFRaBitQ(128, 64, seed=7, device=rank)
    b1.build(X, centroids=C, labels=lab)
    b1.nprobe, b1.k_rerank, b1.probe_split = 12, 40, 1
    d1, i1 = b1.search(Q, 10)
    same.append(np.array_equal(i1, i) and np.array_equal(d1.view(np.uint32), d.view(np.uint32)))
    try:
        b1.build(X)
        same.append(False)
    except RuntimeError:
        same.append(True)
    b2 = ShardedIndexIVFRaBitQ(128, 64, seed=7, device=rank, kmeans_iters=4)
    b2.build(X)
    b3 = ShardedIndexIVFRaBitQ(128, 64, seed=7, device=rank, kmeans_iters=4)
    b3.train(X)
    b3.add(X)
    for b in (b2, b3):
        b.nprobe, b.k_rerank, b.probe_split = 12, 40, 1
    d2, i2 = b2.search(Q, 10)
    d3, i3 = b3.search(Q, 10)
    same.append(np.array_equal(i2, i3) and np.array_equal(d2.view(np.uint32), d3.view(np.uint32)))
    if rank == 0:
        with open(os.path.join(outdir, "res.pkl"), "wb") as f:
            pickle.dump((d, i, C, lab, idx.local.rotation(), idx.local.query_scale, X, Q, idx.local.list_owners(),
                         [s.cpu().numpy() for s in stats], same, dl, il, [s.cpu().numpy() for s in stats_l]), f)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(_ngpu() < 2, reason="needs 2 GPUs")
def test_two_gpu_sharded_search_matches_oracle(oracle):
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_rank_main, args=(2, _port(), td), nprocs=2, join=True)
        d, i, C, lab, P, t4, X, Q, owners, stats, same, dl, il, stats_l = pickle.load(
            open(os.path.join(td, "res.pkl"), "rb"))
    assert same == [True, True, True], same  # build() == train() / centroids + add(); rebuild refused
    oix = oracle.build(X, C, lab, P, t4)
    want = oracle.list_owners("balanced", np.bincount(lab, minlength=64), 2)
    assert np.array_equal(owners, want)  # the default policy of the sharded index
    parts = [oracle.search(oix, Q, 10, 12, 40, shard_rank=r, shard_count=2, slices=1, exchange=True, owner=want,
                           with_stats=True) for r in range(2)]
    for r in range(2):  # vectors scanned / admitted per shard: the shared threshold is the owner's
        assert np.array_equal(stats[r], parts[r][2]), (r, stats[r], parts[r][2])
    want_i, want_d = oracle.merge_candidates([(p[1], p[0]) for p in parts], 10)
    assert np.array_equal(i, want_i)
    assert np.array_equal(d.view(np.uint32), want_d.view(np.uint32))
    parts = [oracle.search(oix, Q, 10, 12, 40, shard_rank=r, shard_count=2, slices=1, exchange=True, owner=want,
                           with_stats=True, scan_kind=2) for r in range(2)]
    for r in range(2):
        assert np.array_equal(stats_l[r], parts[r][2]), (r, stats_l[r], parts[r][2])
    want_i, want_d = oracle.merge_candidates([(p[1], p[0]) for p in parts], 10)
    assert np.array_equal(il, want_i)
    assert np.array_equal(dl.view(np.uint32), want_d.view(np.uint32))
