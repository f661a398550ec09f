"""List-sharded search across ranks, on CPU with gloo (world size 2).

Each rank runs the oracle's sharded search for its own lists (l % 2 == rank), the per-rank
[nq, k] results travel through the product's single all-gather of 8-byte result keys
(neurosamble_b200.sharded.gather_result_keys), and rank 0 merges them by (distance, id).  The
merged result must equal the merge computed without any collective, and every rank must
receive identical bytes.  A second test makes a rank leave before the collective: the other
rank's all-gather must fail within the process group's short timeout (failure detected on
the host, nothing waits forever)."""
import os
import pickle
import socket
import tempfile
from datetime import timedelta

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _merge(dists, ids, k):
    out_d, out_i = [], []
    for q in range(dists.shape[1]):
        keys = []
        for r in range(dists.shape[0]):
            keys += [(float(dists[r, q, j]), int(ids[r, q, j])) for j in range(k) if ids[r, q, j] >= 0]
        keys.sort()
        keys = keys[:k] + [(float("inf"), -1)] * (k - min(k, len(keys)))
        out_d.append([d for d, _ in keys])
        out_i.append([i for _, i in keys])
    return np.array(out_d, np.float32), np.array(out_i, np.int64)


class _KeyPacker:
    """The packing stage of LibStages (rbq_pack_results), restated on CPU tensors."""

    def __init__(self, O):
        self.O = O

    def pack(self, d, ids, keys):
        import torch
        keys.copy_(torch.from_numpy(self.O._keys(ids.numpy(), d.numpy()).view(np.int64)))


def _unkey(keys):
    kk = np.ascontiguousarray(keys).view(np.uint64)
    empty = kk == np.uint64(0xFFFFFFFFFFFFFFFF)
    ids = np.where(empty, -1, (kk & np.uint64(0xFFFFFFFF)).astype(np.int64))
    ob = (kk >> np.uint64(32)).astype(np.uint32)
    d = np.where(empty, np.inf, np.where(ob & 0x80000000, ob & 0x7FFFFFFF, ~ob).astype(np.uint32).view(np.float32))
    return d.astype(np.float32), ids


def _worker(rank, world, port, outdir):
    import torch
    import torch.distributed as dist

    from conftest import mixture
    from oracle import oracle as O
    from neurosamble_b200.sharded import gather_result_keys

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    X, Q = mixture(4000, 64, 12, 0.3, 25, seed=5)
    P, t4 = O.make_rotation(64, 3), O.query_scale(64, 3)
    C, lab = O.kmeans(X, 16, iters=3)
    ix = O.build(X, C, lab, P, t4)
    d, i = O.search(ix, Q, 10, 6, 30, shard_rank=rank, shard_count=world)
    kall = gather_result_keys(_KeyPacker(O), torch.from_numpy(d), torch.from_numpy(i))
    gd, gi = _unkey(kall.numpy())
    with open(os.path.join(outdir, f"rank{rank}.pkl"), "wb") as f:
        pickle.dump({"local": (d, i), "gathered": (gd, gi)}, f)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_results_gather_and_merge_over_gloo():
    world = 2
    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_worker, args=(world, _free_port(), td), nprocs=world, join=True)
        res = [pickle.load(open(os.path.join(td, f"rank{r}.pkl"), "rb")) for r in range(world)]
    locals_d = np.stack([r["local"][0] for r in res])
    locals_i = np.stack([r["local"][1] for r in res])
    for r in res:  # every rank holds every rank's block, in rank order
        assert np.array_equal(r["gathered"][1], locals_i)
        assert np.array_equal(r["gathered"][0].view(np.uint32), locals_d.view(np.uint32))
    md, mi = _merge(locals_d, locals_i, 10)
    # shard ownership: rank r only returns ids whose list is r (mod 2)
    assert (mi >= 0).all()
    gd, gi = _merge(res[0]["gathered"][0], res[0]["gathered"][1], 10)
    assert np.array_equal(gi, mi)


def _leaver(rank, world, port, outdir):
    import torch
    import torch.distributed as dist

    from oracle import oracle as O
    from neurosamble_b200.sharded import gather_result_keys

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=4))
    if rank == 1:
        return  # leaves between steps: never joins the collective
    err = ""
    try:
        gather_result_keys(_KeyPacker(O), torch.zeros((3, 2)), torch.zeros((3, 2), dtype=torch.int64))
    except Exception as e:  # noqa: BLE001
        err = type(e).__name__ + ": " + str(e)[:200]
    with open(os.path.join(outdir, "rank0.txt"), "w") as f:
        f.write(err)


def test_missing_rank_fails_the_collective_within_the_timeout():
    with tempfile.TemporaryDirectory() as td:
        ctx = mp.start_processes(_leaver, args=(2, _free_port(), td), nprocs=2, join=False, start_method="spawn")
        ctx.join(timeout=120)
        for p in ctx.processes:
            if p.is_alive():
                p.terminate()
        err = open(os.path.join(td, "rank0.txt")).read()
    assert err, "rank 0's all-gather returned although rank 1 never joined"


class _OracleStages:
    """The stage interface of neurosamble_b200.sharded.LibStages, computed by the CPU oracle on
    CPU tensors: lets the product's sharded orchestration (front-end split, record all-gather,
    seed all-reduce, result all-gather) run over gloo without a GPU."""

    def __init__(self, O, ix, rank, world, owner=None):
        self.O, self.ix, self.rank, self.world, self.owner = O, ix, rank, world, owner

    def rotate(self, q, qr):
        import torch
        qr.copy_(torch.from_numpy(self.O.rotate(q.numpy(), self.ix.P)))

    def prep(self, qr, planes, delta, k1):
        import torch
        bits = planes.shape[1]
        pl, de, kk, _ = self.O.query_prep(qr.numpy(), self.ix.t4 if bits == 4 else self.ix.t8, bits)
        planes.copy_(torch.from_numpy(np.ascontiguousarray(pl).view(np.int32).reshape(planes.shape)))
        delta.copy_(torch.from_numpy(de))
        k1.copy_(torch.from_numpy(kk))

    def coarse(self, qr, margin, probes, g):
        import torch
        p, gg = self.O.coarse(qr.numpy(), self.ix.c_rot, probes.shape[1])
        probes.copy_(torch.from_numpy(p))
        g.copy_(torch.from_numpy(gg))

    def bound_seed(self, qr, planes, delta, k1, probes, g, R, cap, tau):
        import torch
        t = self.O.bound_seed(self.ix, planes.numpy().view(np.uint32), delta.numpy(), k1.numpy(), probes.numpy(),
                              g.numpy(), R, shard_rank=self.rank, shard_count=self.world, owner=self.owner)
        tau.copy_(torch.from_numpy(t))

    def scan(self, qr, planes, delta, k1, probes, g, tau0, init, R, prune, slices, cap, ids, d, stats, mode=0):
        import torch
        oi, od = self.O.scan(self.ix, qr.numpy(), planes.numpy().view(np.uint32), delta.numpy(), k1.numpy(),
                             probes.numpy(), g.numpy(), R, cap=cap, prune=prune, slices=slices,
                             shard_rank=self.rank, shard_count=self.world,
                             tau0=tau0.numpy() if tau0 is not None else None,
                             init=(init[0].numpy(), init[1].numpy()) if init is not None else None,
                             owner=self.owner, mode=mode or None)
        ids.copy_(torch.from_numpy(oi))
        d.copy_(torch.from_numpy(od))

    def bound_seed_owned(self, qr, planes, delta, k1, probes, g, R, cap, tau):
        import torch
        t = self.O.bound_seed(self.ix, planes.numpy().view(np.uint32), delta.numpy(), k1.numpy(), probes.numpy(),
                              g.numpy(), R, shard_rank=self.rank, shard_count=self.world, owner=self.owner)
        p0 = probes.numpy()[:, 0]
        own0 = self.owner[p0] if self.owner is not None else p0 % self.world
        tau.copy_(torch.from_numpy(np.where(own0 == self.rank, t, np.float32(np.inf)).astype(np.float32)))

    def scan_lists(self, qr, planes, delta, k1, probes, g, tau0, R, ids, d, stats):
        import torch
        oi, od = self.O.list_scan(self.ix, qr.numpy(), planes.numpy().view(np.uint32), delta.numpy(), k1.numpy(),
                                  probes.numpy(), g.numpy(), R, tau0.numpy(), shard_rank=self.rank,
                                  shard_count=self.world, owner=self.owner)
        ids.copy_(torch.from_numpy(oi))
        d.copy_(torch.from_numpy(od))

    def merge(self, d, ids, out_d, out_i):
        import torch
        mi, md = self.O.merge_candidates([(ids[p].numpy(), d[p].numpy()) for p in range(d.shape[0])], d.shape[2])
        out_d.copy_(torch.from_numpy(md))
        out_i.copy_(torch.from_numpy(mi))

    def pack(self, d, ids, keys):
        import torch
        keys.copy_(torch.from_numpy(self.O._keys(ids.numpy(), d.numpy()).view(np.int64)))

    def merge_keys(self, keys, out_d, out_i):
        import torch
        kk = keys.numpy().view(np.uint64)
        empty = kk == np.uint64(0xFFFFFFFFFFFFFFFF)
        ids = np.where(empty, -1, (kk & np.uint64(0xFFFFFFFF)).astype(np.int64))
        ob = (kk >> np.uint64(32)).astype(np.uint32)
        d = np.where(empty, np.inf, np.where(ob & 0x80000000, ob & 0x7FFFFFFF, ~ob).astype(np.uint32).view(np.float32))
        self.merge(torch.from_numpy(d.astype(np.float32)), torch.from_numpy(ids), out_d, out_i)

    def rerank(self, q, cand, k, out_d, out_i):
        import torch
        dd, ii = self.O.rerank(self.ix.X, q.numpy(), cand.numpy(), k)
        out_d.copy_(torch.from_numpy(dd))
        out_i.copy_(torch.from_numpy(ii))


def _seeded_worker(rank, world, port, outdir, nq, prune, policy, bits, bpd, kind):
    import torch
    import torch.distributed as dist

    from conftest import mixture
    from oracle import oracle as O
    from neurosamble_b200.sharded import sharded_search

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    X, Q = mixture(6000, 64, 12, 0.3, 40, seed=9)
    Q = Q[:nq]
    P, t4 = O.make_rotation(64, 3), O.query_scale(64, 3)
    C, lab = O.kmeans(X, 24, iters=3)
    ix = O.build(X, C, lab, P, t4, bits_per_dim=bpd)
    ix.t8 = O.query_scale(64, 3, 7)
    owner = O.list_owners(policy, np.bincount(lab, minlength=24), world)
    d, i = sharded_search(_OracleStages(O, ix, rank, world, owner), torch.from_numpy(Q), 10, 8, 60, prune, 0, 0, 0,
                          64, rank, world, query_bits=bits, nlist=24, scan_kind=kind)
    with open(os.path.join(outdir, f"rank{rank}.pkl"), "wb") as f:
        pickle.dump((d.numpy(), i.numpy()), f)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,nq,prune,policy,bits,bpd,kind", [
    (2, 40, 1, "balanced", 4, 1, 0), (3, 7, 1, "round_robin", 4, 1, 0), (2, 40, 0, "balanced", 4, 1, 0),
    (2, 40, 1, "balanced", 8, 1, 0), (2, 40, 1, "balanced", 16, 1, 0), (3, 9, 1, "round_robin", 32, 1, 0),
    (2, 40, 1, "balanced", 4, 4, 0), (3, 9, 1, "round_robin", 16, 3, 0),
    (2, 40, 1, "balanced", 4, 1, 2), (3, 9, 1, "round_robin", 8, 1, 2), (2, 40, 1, "balanced", 4, 3, 2)])
def test_seeded_sharded_search_over_gloo(world, nq, prune, policy, bits, bpd, kind):
    """The orchestration (queries split for the rotation and coarse quantiser and padded, rotated
    rows and probe rows all-gathered, seeds all-reduced, results all-gathered and merged) gives, on every rank, the
    merge of the oracle's per-shard searches with the shared seed.  With the prune off every
    shard keeps its exact top-R by estimate, so the shards' candidates contain the single-shard
    top-R and the reranked distances are, rank by rank, no larger than the single-shard's."""
    from conftest import mixture
    from oracle import oracle as O
    from neurosamble_b200.sharded import plan

    with tempfile.TemporaryDirectory() as td:
        mp.spawn(_seeded_worker, args=(world, _free_port(), td, nq, prune, policy, bits, bpd, kind), nprocs=world,
                 join=True)
        res = [pickle.load(open(os.path.join(td, f"rank{r}.pkl"), "rb")) for r in range(world)]
    X, Q = mixture(6000, 64, 12, 0.3, 40, seed=9)
    Q = Q[:nq]
    P, t4 = O.make_rotation(64, 3), O.query_scale(64, 3)
    C, lab = O.kmeans(X, 24, iters=3)
    ix = O.build(X, C, lab, P, t4, bits_per_dim=bpd)
    ix.t8 = O.query_scale(64, 3, 7)
    slices = plan(nq, 8, 10, 60, 0, 0, world)[1]
    owner = O.list_owners(policy, np.bincount(lab, minlength=24), world)
    parts = [O.search(ix, Q, 10, 8, 60, prune=prune, slices=slices, shard_rank=r, shard_count=world, exchange=True,
                      owner=owner, query_bits=bits, scan_kind=kind) for r in range(world)]
    want_i, want_d = O.merge_candidates([(p[1], p[0]) for p in parts], 10)
    for d, i in res:
        assert np.array_equal(i, want_i)
        assert np.array_equal(d.view(np.uint32), want_d.view(np.uint32))
    if not prune:
        d1, i1 = O.search(ix, Q, 10, 8, 60, prune=0)
        assert (want_d <= d1).all()
        assert np.mean([len(set(a) & set(b)) for a, b in zip(want_i.tolist(), i1.tolist())]) >= 9.5
