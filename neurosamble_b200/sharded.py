"""List-sharded IVF-RaBitQ over the GPUs of one box: one process per GPU.

Every list lives on one rank (every rank keeps the full centroid table, rotation and t4):
"balanced" (the default) spreads the lists by size^2 when the first batch is added, so that
each rank's scan work is about equal; "round_robin" puts list l on rank l % world.
A search of a batch replicated on every rank runs in four steps:

1. front end: rank r rotates and coarse-quantises queries [r*nl, (r+1)*nl)
   (nl = ceil(nq / world)); two all-gathers hand every rank the rotated queries and the
   [probes | g] rows of the whole batch, which every rank then 4-bit-quantises (cheap);
2. seed: each rank computes the bound seed (the R-th smallest RaBitQ upper bound) of the
   nearest probed list of the queries whose nearest list it owns; an all-reduce (min) gives
   every rank that threshold, so a shard prunes its lists as tightly as one GPU prunes all of
   them (without it a shard far from the query admits most of its vectors);
3. scan the shard's probed lists from that threshold and rerank the shard's candidates (only
   those under the threshold survive, ~R / world per shard).  Large batches take the list scan
   instead (the library's rule, scan_kind): the bound seed over the leading owned lists of the
   nearest probe's owner, all-reduced (min); the tile scan of the nearest probe on its owner from
   that seed; the
   nearest list's R-th distance, all-reduced (min), as the fixed threshold of the list scan of
   every rank's other probes;
4. the per-rank [nq, k] results cross NVLink in one all-gather (one packed buffer per rank)
   and are merged on the device by (distance, id).

The reference RaBitQ path is single-GPU (src/rabitq_gpu/rabitq_search.cu:11); the sharding
follows FAISS's sharded GPU search that map_full.py:302-317 uses for IVF-Flat.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .index import IndexIVFRaBitQ, _ptr, _stream_ptr

SCAN_TILE = _lib.lib().rbq_scan_tile()  # vectors per scan tile (kScanTile in the library)


def _pow2(v: int) -> int:
    p = 1
    while p < v:
        p <<= 1
    return p


def uses_list_scan(scan_kind: int, query_bits: int, prune: bool, dp: int, nq: int, nprobe: int, nlist: int,
                   n_total: int = 0, R: int = 0) -> bool:
    """The library's choice of scan (rbq_search_params_t.scan_kind): 2 the list scan, 1 the tile
    scan, 0 the list scan for popcount modes with the prune on when nq * nprobe >= 64 nlist and
    the index holds n_total >= R nlist vectors."""
    able = query_bits in (4, 8) and prune and dp % 32 == 0 and dp <= 768
    if scan_kind == 2:
        if not able:
            raise RuntimeError("list scan: needs QUANT4 / QUANT8, the prune on and a padded dim <= 768")
        return True
    return scan_kind == 0 and able and nlist > 0 and nq * nprobe >= 64 * nlist and n_total >= R * nlist


def plan(nq: int, nprobe: int, k: int, k_rerank: int, probe_split: int, cand_cap: int, world: int):
    """(R, slices, cap) of a sharded search: the library's search planning (plan_search)."""
    R = max(k_rerank, k) if k_rerank > 0 else k
    own = max(1, (nprobe + world - 1) // world)
    sl = probe_split if probe_split > 0 else max(1, 512 // max(1, nq))
    sl = max(1, min(sl, own, max(1, 8192 // R)))
    cap = max(_pow2(cand_cap if cand_cap > 0 else 1024), _pow2(R + SCAN_TILE))
    return R, sl, cap


def gather_result_keys(stages, dist_t: torch.Tensor, ids_t: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather every rank's [nq, k] results with a single collective, each result packed as
    one 8-byte key ((order-preserving distance bits) << 32 | id): [world, nq, k] int64."""
    world = dist.get_world_size(group)
    nq, k = dist_t.shape
    keys = torch.empty((nq, k), dtype=torch.int64, device=dist_t.device)
    stages.pack(dist_t, ids_t, keys)
    out = torch.empty((world * nq, k), dtype=torch.int64, device=dist_t.device)
    dist.all_gather_into_tensor(out, keys, group=group)
    return out.view(world, nq, k)


class ShardedIndexIVFRaBitQ:
    """The IndexIVFRaBitQ API over `world` ranks of a process group (NCCL)."""

    def __init__(self, d: int, nlist: int, seed: int = 7, group=None, device: int | None = None,
                 shard_policy: str = "balanced", **kw):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.d, self.nlist = d, nlist
        self.local = IndexIVFRaBitQ(d, nlist, seed=seed, device=device, shard_rank=self.rank,
                                    shard_count=self.world, shard_policy=shard_policy, **kw)
        self.device = self.local.device

    def __getattr__(self, name):
        if name in ("nprobe", "k_rerank", "prune", "probe_split", "cand_cap", "coarse_margin", "query_bits",
                    "scan_kind"):
            return getattr(self.local, name)
        raise AttributeError(name)

    def __setattr__(self, name, value):
        if name in ("nprobe", "k_rerank", "prune", "probe_split", "cand_cap", "coarse_margin", "query_bits",
                    "scan_kind"):
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

    def build(self, x, centroids=None, labels=None) -> None:
        """train (or the given centroids, on every rank) + add, as IndexIVFRaBitQ.build; like
        rbq_build it refuses an index that already holds vectors."""
        if self.ntotal != 0:
            raise RuntimeError("build: the index already holds vectors (use add)")
        if centroids is None:
            if labels is not None:
                raise RuntimeError("build: labels need the centroids they refer to")
            self.train(x)
        else:
            self.local.set_centroids(centroids)
        self.add(x, labels)

    def search_local(self, x, k: int):
        t, _ = self.local._to_device(x)
        d, i = self.local.search(t, k)
        return d, i

    def search(self, x, k: int, stats: torch.Tensor | None = None, timings: dict | None = None):
        """(D [nq, k], I [nq, k]) of the whole index for a batch every rank passes.

        stats (optional int64[2] on this rank's device) accumulates this rank's vectors
        scanned / admitted by the prune; timings (optional dict) receives this rank's
        milliseconds per stage."""
        t, on_dev = self.local._to_device(x)
        if self.world == 1:
            d, i = self.local.search(t, k)
        else:
            loc = self.local
            d, i = sharded_search(LibStages(loc), t, int(k), int(loc.nprobe), int(loc.k_rerank), bool(loc.prune),
                                  int(loc.probe_split), int(loc.cand_cap), int(loc.coarse_margin),
                                  loc.info().padded_dim, self.rank, self.world, self.group, stats,
                                  query_bits=int(loc.query_bits), timings=timings, nlist=self.nlist,
                                  scan_kind=int(loc.scan_kind), n_total=self.ntotal)
            if loc.metric == "ip":
                d = 1.0 - 0.5 * d
        if on_dev:
            return d, i
        return d.cpu().numpy(), i.cpu().numpy()


class LibStages:
    """The stage entry points of librbq.so on one index (CUDA tensors, the index's stream)."""

    def __init__(self, index: IndexIVFRaBitQ):
        self.h = index.handle
        self.device = index.device
        self.st = _stream_ptr(index.device)

    def rotate(self, q, qr):
        with torch.cuda.device(self.device):
            _lib.call("rbq_rotate", self.h, _ptr(q), q.shape[0], _ptr(qr), self.st)

    def prep(self, qr, planes, delta, k1):
        """planes: [nq, bits, W]; bits (4 or 8) is the query code width."""
        with torch.cuda.device(self.device):
            _lib.call("rbq_query_prep", self.h, _ptr(qr), qr.shape[0], _ptr(planes), _ptr(delta), _ptr(k1),
                      planes.shape[1], self.st)

    def coarse(self, qr, margin, probes, g):
        with torch.cuda.device(self.device):
            _lib.call("rbq_coarse", self.h, _ptr(qr), qr.shape[0], probes.shape[1], margin, _ptr(probes), _ptr(g),
                      self.st)

    def bound_seed(self, qr, planes, delta, k1, probes, g, R, cap, tau):
        assert probes.stride(1) == 1 and g.stride() == probes.stride()
        with torch.cuda.device(self.device):
            _lib.call("rbq_bound_seed", self.h, _ptr(qr), _ptr(planes), _ptr(delta), _ptr(k1), qr.shape[0],
                      _ptr(probes), _ptr(g), probes.shape[1], probes.stride(0), R, cap, _ptr(tau), planes.shape[1],
                      self.st)

    def scan(self, qr, planes, delta, k1, probes, g, tau0, init, R, prune, slices, cap, ids, d, stats, mode=0):
        """probes / g: [nq, p] views with unit column stride and one row stride; mode 16 / 32
        scans by LUT16 / LUT32 tables (default: the planes' code width)."""
        assert probes.stride(1) == 1 and g.stride() == probes.stride()
        with torch.cuda.device(self.device):
            _lib.call("rbq_scan", self.h, _ptr(qr), _ptr(planes), _ptr(delta), _ptr(k1), qr.shape[0], _ptr(probes),
                      _ptr(g), probes.shape[1], probes.stride(0), _ptr(tau0) if tau0 is not None else None,
                      _ptr(init[0]) if init is not None else None, _ptr(init[1]) if init is not None else None, R,
                      prune, slices, cap, _ptr(ids), _ptr(d), _ptr(stats) if stats is not None else None,
                      mode or planes.shape[1], self.st)

    def bound_seed_owned(self, qr, planes, delta, k1, probes, g, R, cap, tau):
        """bound_seed for the queries whose nearest probe this rank owns (+inf elsewhere)."""
        assert probes.stride(1) == 1 and g.stride() == probes.stride()
        with torch.cuda.device(self.device):
            _lib.call("rbq_bound_seed_owned", self.h, _ptr(qr), _ptr(planes), _ptr(delta), _ptr(k1), qr.shape[0],
                      _ptr(probes), _ptr(g), probes.shape[1], probes.stride(0), R, cap, _ptr(tau), planes.shape[1],
                      self.st)

    def scan_lists(self, qr, planes, delta, k1, probes, g, tau0, R, ids, d, stats):
        """The list scan with fixed thresholds tau0 (rbq_scan_lists); probes / g as in scan."""
        assert probes.stride(1) == 1 and g.stride() == probes.stride()
        with torch.cuda.device(self.device):
            _lib.call("rbq_scan_lists", self.h, _ptr(qr), _ptr(planes), _ptr(delta), _ptr(k1), qr.shape[0],
                      _ptr(probes), _ptr(g), probes.shape[1], probes.stride(0), _ptr(tau0), R, _ptr(ids), _ptr(d),
                      _ptr(stats) if stats is not None else None, planes.shape[1], self.st)

    def merge(self, d, ids, out_d, out_i):
        with torch.cuda.device(self.device):
            _lib.call("rbq_merge_results", _ptr(d), _ptr(ids), d.shape[0], d.shape[1], d.shape[2], _ptr(out_d),
                      _ptr(out_i), self.st)

    def pack(self, d, ids, keys):
        with torch.cuda.device(self.device):
            _lib.call("rbq_pack_results", _ptr(d), _ptr(ids), d.numel(), _ptr(keys), self.st)

    def merge_keys(self, keys, out_d, out_i):
        """keys [parts, nq, k] (rbq_pack_results) -> top-k by (dist, id)."""
        with torch.cuda.device(self.device):
            _lib.call("rbq_merge_result_keys", _ptr(keys), keys.shape[0], keys.shape[1], keys.shape[2], _ptr(out_d),
                      _ptr(out_i), self.st)

    def rerank(self, q, cand, k, out_d, out_i):
        with torch.cuda.device(self.device):
            _lib.call("rbq_rerank", self.h, _ptr(q), q.shape[0], _ptr(cand), cand.shape[1], k, _ptr(out_d),
                      _ptr(out_i), self.st)


class _StageClock:
    """CUDA events at the stage boundaries of one sharded search (timings=dict): after the search,
    timings[stage] = milliseconds on this rank's current stream."""

    def __init__(self, timings, device):
        self.t = timings
        self.ev = []
        self.on = timings is not None and device.type == "cuda"

    def mark(self, name):
        if self.on:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.ev.append((name, e))

    def finish(self):
        if not self.on:
            return
        self.ev[-1][1].synchronize()
        for (_, a), (name, b) in zip(self.ev, self.ev[1:]):
            self.t[name] = self.t.get(name, 0.0) + a.elapsed_time(b)


def sharded_search(stages, t: torch.Tensor, k: int, nprobe: int, k_rerank: int, prune: bool, probe_split: int,
                   cand_cap: int, margin: int, dp: int, rank: int, world: int, group=None, stats=None,
                   query_bits: int = 4, timings=None, nlist: int = 0, scan_kind: int = 0, n_total: int = 0):
    """The four steps of a sharded search (module docstring) for the batch t [nq, D] that
    every rank passes; `stages` computes (LibStages: librbq.so), this function moves data.
    timings (optional dict) receives this rank's milliseconds per stage."""
    dev = t.device
    clk = _StageClock(timings, dev)
    clk.mark("start")
    nq = t.shape[0]
    P = nprobe
    R, slices, cap = plan(nq, P, k, k_rerank, probe_split, cand_cap, world)
    nl = (nq + world - 1) // world
    lo, hi = min(nq, rank * nl), min(nq, (rank + 1) * nl)
    # 1. front end: this rank's queries (padded with copies of the last query) rotated and
    #    coarse-quantised; rotated rows and [probes | g] rows all-gathered; planes of the batch.
    qloc = t[lo:hi]
    if hi - lo < nl:
        qloc = torch.cat([qloc, t[nq - 1:].expand(nl - (hi - lo), t.shape[1])])
    qr_l = torch.empty((nl, dp), dtype=torch.float32, device=dev)
    stages.rotate(qloc.contiguous(), qr_l)
    pl = torch.empty((nl, P), dtype=torch.int32, device=dev)
    gl = torch.empty((nl, P), dtype=torch.float32, device=dev)
    stages.coarse(qr_l, margin, pl, gl)
    clk.mark("front_end (rotate + coarse, own queries)")
    qr_all = torch.empty((world * nl, dp), dtype=torch.float32, device=dev)
    dist.all_gather_into_tensor(qr_all, qr_l, group=group)
    send = torch.cat([pl, gl.view(torch.int32)], dim=1)
    recv = torch.empty((world * nl, 2 * P), dtype=torch.int32, device=dev)
    dist.all_gather_into_tensor(recv, send, group=group)
    clk.mark("all_gather (rotated rows, probes)")
    qr = qr_all[:nq]
    probes, g = recv[:nq, :P], recv[:nq, P:].view(torch.float32)  # row stride 2P
    lut = query_bits in (16, 32)  # LUT16 / LUT32: tables of the float query, no seed
    planes = torch.empty((nq, 8 if query_bits == 8 else 4, dp // 32), dtype=torch.int32, device=dev)
    delta = torch.empty(nq, dtype=torch.float32, device=dev)
    k1 = torch.empty(nq, dtype=torch.float32, device=dev)
    stages.prep(qr, planes, delta, k1)
    clk.mark("query planes")
    if not lut and uses_list_scan(scan_kind, query_bits, prune, dp, nq, P, nlist, n_total, R):
        mi, md = _sharded_list_scan(stages, qr, planes, delta, k1, probes, g, R, cap, stats, group, clk)
        return _finish(stages, t, mi, md, k, k_rerank, group, clk)
    # 2. seed: the bound seed of the nearest probe, on the rank that owns it (+inf elsewhere);
    #    min over ranks.
    tau = None
    if prune and not lut:
        tau = torch.empty(nq, dtype=torch.float32, device=dev)
        stages.bound_seed(qr, planes, delta, k1, probes[:, :1], g[:, :1], R, cap, tau)
        clk.mark("bound seed")
        dist.all_reduce(tau, op=dist.ReduceOp.MIN, group=group)
        clk.mark("all_reduce (seed)")
    # 3. this shard's probed lists from the shared threshold; rerank its candidates.
    mi = torch.empty((nq, R), dtype=torch.int64, device=dev)
    md = torch.empty((nq, R), dtype=torch.float32, device=dev)
    stages.scan(qr, planes, delta, k1, probes, g, tau, None, R, int(prune), slices, cap, mi, md, stats,
                mode=query_bits if lut else 0)
    clk.mark("scan")
    return _finish(stages, t, mi, md, k, k_rerank, group, clk)


def _sharded_list_scan(stages, qr, planes, delta, k1, probes, g, R, cap, stats, group, clk):
    """Step 3 of a large batch: this rank's R best candidates by the list scan (module
    docstring), thresholds shared by two all-reduces (min)."""
    nq, P = probes.shape
    dev = qr.device
    tau = torch.empty(nq, dtype=torch.float32, device=dev)
    stages.bound_seed_owned(qr, planes, delta, k1, probes, g, R, cap, tau)
    clk.mark("bound seed")
    dist.all_reduce(tau, op=dist.ReduceOp.MIN, group=group)
    clk.mark("all_reduce (seed)")
    d2 = torch.empty((2, nq, R), dtype=torch.float32, device=dev)
    i2 = torch.empty((2, nq, R), dtype=torch.int64, device=dev)
    stages.scan(qr, planes, delta, k1, probes[:, :1], g[:, :1], tau, None, R, 1, 1, cap, i2[0], d2[0], stats)
    if P == 1:
        clk.mark("scan")
        return i2[0], d2[0]
    tau1 = torch.where(i2[0][:, R - 1] >= 0, torch.minimum(tau, d2[0][:, R - 1]), tau).contiguous()
    dist.all_reduce(tau1, op=dist.ReduceOp.MIN, group=group)
    clk.mark("scan (nearest probe) + all_reduce (threshold)")
    stages.scan_lists(qr, planes, delta, k1, probes[:, 1:], g[:, 1:], tau1, R, i2[1], d2[1], stats)
    mi = torch.empty((nq, R), dtype=torch.int64, device=dev)
    md = torch.empty((nq, R), dtype=torch.float32, device=dev)
    stages.merge(d2, i2, md, mi)
    clk.mark("scan")
    return mi, md


def _finish(stages, t, mi, md, k, k_rerank, group, clk):
    """Steps 3 (rerank) and 4 of a sharded search from this rank's candidates (mi, md)."""
    dev = t.device
    nq = t.shape[0]
    if k_rerank > 0:
        d = torch.empty((nq, k), dtype=torch.float32, device=dev)
        i = torch.empty((nq, k), dtype=torch.int64, device=dev)
        stages.rerank(t, mi, k, d, i)
    else:
        d, i = md[:, :k].contiguous(), mi[:, :k].contiguous()
    clk.mark("rerank")
    # 4. one all-gather of the per-rank top-k (8-byte keys), merged by (distance, id).
    kall = gather_result_keys(stages, d, i, group)
    clk.mark("all_gather (results)")
    out_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
    out_i = torch.empty((nq, k), dtype=torch.int64, device=dev)
    stages.merge_keys(kall, out_d, out_i)
    clk.mark("merge")
    clk.finish()
    return out_d, out_i
