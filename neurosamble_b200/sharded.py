"""List-sharded IVF-RaBitQ over the GPUs of one box: one process per GPU.

List l lives on rank l % world (every rank keeps the full centroid table, rotation and t4).
A search runs the full coarse quantiser on every rank, scans only the rank's own probed
lists, reranks its local top-R, and returns a local top-k; the per-rank [nq, k] results
cross NVLink in ONE all-gather (one packed buffer per rank) and are merged on the device
by (distance, id).  The reference RaBitQ path is single-GPU (src/rabitq_gpu/rabitq_search.cu:11);
the sharding follows FAISS's sharded GPU search that map_full.py:302-317 uses for IVF-Flat.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .index import IndexIVFRaBitQ, _ptr, _stream_ptr


def pack_results(dist_t: torch.Tensor, ids_t: torch.Tensor) -> torch.Tensor:
    """One byte buffer per rank: [dist f32 (nq*k) | pad to 16 B | ids i64 (nq*k)]."""
    n = dist_t.numel()
    off = (n * 4 + 15) // 16 * 16
    buf = torch.empty(off + n * 8, dtype=torch.uint8, device=dist_t.device)
    buf[: n * 4].view(torch.float32).copy_(dist_t.reshape(-1))
    buf[off: off + n * 8].view(torch.int64).copy_(ids_t.reshape(-1))
    return buf


def unpack_gathered(out: torch.Tensor, world: int, nq: int, k: int):
    """[world * bytes] gathered buffers -> (dist [world, nq, k], ids [world, nq, k])."""
    n = nq * k
    off = (n * 4 + 15) // 16 * 16
    per = out.view(world, -1)
    d = per[:, : n * 4].contiguous().view(torch.float32).view(world, nq, k)
    i = per[:, off: off + n * 8].contiguous().view(torch.int64).view(world, nq, k)
    return d, i


def gather_results(dist_t: torch.Tensor, ids_t: torch.Tensor, group=None):
    """All-gather every rank's [nq, k] results with a single collective."""
    world = dist.get_world_size(group)
    buf = pack_results(dist_t, ids_t)
    out = torch.empty(world * buf.numel(), dtype=torch.uint8, device=buf.device)
    dist.all_gather_into_tensor(out, buf, group=group)
    return unpack_gathered(out, world, dist_t.shape[0], dist_t.shape[1])


def merge_results(dist_all: torch.Tensor, ids_all: torch.Tensor):
    """[parts, nq, k] on a CUDA device -> [nq, k] by (distance, id), in librbq.so."""
    parts, nq, k = dist_all.shape
    dev = dist_all.device.index
    out_d = torch.empty((nq, k), dtype=torch.float32, device=dist_all.device)
    out_i = torch.empty((nq, k), dtype=torch.int64, device=dist_all.device)
    with torch.cuda.device(dev):
        _lib.call("rbq_merge_results", _ptr(dist_all.contiguous()), _ptr(ids_all.contiguous()), parts, nq, k,
                  _ptr(out_d), _ptr(out_i), _stream_ptr(dev))
    return out_d, out_i


class ShardedIndexIVFRaBitQ:
    """The IndexIVFRaBitQ API over `world` ranks of a process group (NCCL)."""

    def __init__(self, d: int, nlist: int, seed: int = 7, group=None, device: int | None = None, **kw):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.d, self.nlist = d, nlist
        self.local = IndexIVFRaBitQ(d, nlist, seed=seed, device=device, shard_rank=self.rank,
                                    shard_count=self.world, **kw)
        self.device = self.local.device

    def __getattr__(self, name):
        if name in ("nprobe", "k_rerank", "prune", "probe_split", "cand_cap", "coarse_margin"):
            return getattr(self.local, name)
        raise AttributeError(name)

    def __setattr__(self, name, value):
        if name in ("nprobe", "k_rerank", "prune", "probe_split", "cand_cap", "coarse_margin"):
            setattr(self.local, name, value)
        else:
            object.__setattr__(self, name, value)

    @property
    def ntotal(self) -> int:
        return self.local.ntotal

    def train(self, x) -> None:
        """Rank 0 trains; the centroids are broadcast so every rank holds the same table."""
        src = dist.get_global_rank(self.group, 0) if self.group is not None else 0
        C = torch.empty((self.nlist, self.d), dtype=torch.float32, device=f"cuda:{self.device}")
        if self.rank == 0:
            self.local.train(x)
            C.copy_(torch.from_numpy(self.local.centroids()[0]))
        dist.broadcast(C, src=src, group=self.group)
        if self.rank != 0:
            self.local.set_centroids(C.cpu().numpy())

    def add(self, x, labels=None) -> None:
        """Every rank passes the same rows; each keeps the rows of its own lists."""
        self.local.add(x, labels)

    def search_local(self, x, k: int):
        t, _ = self.local._to_device(x)
        d, i = self.local.search(t, k)
        return d, i

    def search(self, x, k: int):
        t, on_dev = self.local._to_device(x)
        d, i = self.local.search(t, k)
        if self.world > 1:
            dall, iall = gather_results(d, i, self.group)
            d, i = merge_results(dall, iall)
        if on_dev:
            return d, i
        return d.cpu().numpy(), i.cpu().numpy()
