"""List-sharded search across ranks, on CPU with gloo (world size 2).

Each rank runs the oracle's sharded search for its own lists (l % 2 == rank), the per-rank
[nq, k] results travel through the product's single-buffer all-gather
(neurosamble_b200.sharded.gather_results), and rank 0 merges them by (distance, id).  The
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


def _worker(rank, world, port, outdir):
    import torch
    import torch.distributed as dist

    from conftest import mixture
    from oracle import oracle as O
    from neurosamble_b200.sharded import gather_results

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    X, Q = mixture(4000, 64, 12, 0.3, 25, seed=5)
    P, t4 = O.make_rotation(64, 3), O.query_scale(64, 3)
    C, lab = O.kmeans(X, 16, iters=3)
    ix = O.build(X, C, lab, P, t4)
    d, i = O.search(ix, Q, 10, 6, 30, shard_rank=rank, shard_count=world)
    gd, gi = gather_results(torch.from_numpy(d), torch.from_numpy(i))
    with open(os.path.join(outdir, f"rank{rank}.pkl"), "wb") as f:
        pickle.dump({"local": (d, i), "gathered": (gd.numpy(), gi.numpy())}, f)
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

    from neurosamble_b200.sharded import gather_results

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=4))
    if rank == 1:
        return  # leaves between steps: never joins the collective
    err = ""
    try:
        gather_results(torch.zeros((3, 2)), torch.zeros((3, 2), dtype=torch.int64))
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
