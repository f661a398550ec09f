#!/usr/bin/env python
"""Benchmark: queries/sec of IVF-RaBitQ search on benchmark config 2 (1M x 256, nlist 1024,
nprobe 32, k 10, exact rerank, query batch 10,000), 1..8 B200 with lists sharded per GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2|4|5]

One step = one search of one query batch.  `value` times the batch with queries resident
in HBM (CUDA events, L2 flushed before every step); `e2e` times the C-ABI call with host
buffers (rbq_search_host: H2D of the queries, search, D2H of distances and ids).  Under
torchrun (N > 1) the lists are spread over the ranks by size (each list on one rank), every
rank scans its own lists, and the per-rank results are merged after one NCCL all-gather; times
are the max over ranks.  `--impl reference` times the CPU restatement of the reference search
(oracle/, all host cores; the tile scan, the reference's own algorithm) on the same workload.  `--config 4` / `--config 5` run the benchmark's
100M x 128 (nlist 65,536) and 20M x 768 (nlist 16,384) configurations with data generated on
the device and recall measured on a 1,000-query sample (supplementary lines; no CPU baseline).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import threading
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

# Benchmark config 2 (the metric's configuration), and configs 4 and 5 (supplementary).
CFG = dict(n=1_000_000, d=256, centres=4096, sigma=0.25, nq=10_000, qsigma=0.05, nlist=1024, nprobe=32, k=10,
           rerank=100, seed=2024, config=2, aniso=0, device_data=False, gt_sample=10_000)
CONFIGS = {
    2: CFG,
    3: dict(n=200_000, d=256, centres=0, sigma=0.0, nq=200_000, qsigma=0.0, nlist=2048, nprobe=48, k=20,
            rerank=200, seed=3003, config=3, aniso=0, device_data=True, gt_sample=10_000, generator="reads",
            genome_len=10_000_000, read_len=5000),
    4: dict(n=100_000_000, d=128, centres=65536, sigma=0.3, nq=100_000, qsigma=0.05, nlist=65536, nprobe=64,
            k=100, rerank=400, seed=4004, config=4, aniso=0, device_data=True, gt_sample=1000),
    5: dict(n=20_000_000, d=768, centres=16384, sigma=0.2, nq=50_000, qsigma=0.05, nlist=16384, nprobe=128,
            k=50, rerank=500, seed=5005, config=5, aniso=1, device_data=True, gt_sample=1000),
}
RERANK_LADDER = (100, 150, 200, 300, 400, 600, 800)


def rerank_ladder(cfg):
    """Rerank depths tried in order until recall reaches the target.  Extra-bit codes estimate
    closely enough that no rerank (0, the reference's own output) or a short one may do."""
    if cfg.get("bits_per_dim", 1) > 1:
        return (0, 20, 50) + RERANK_LADDER
    return RERANK_LADDER
RECALL_TARGET = 0.95
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def make_data(cfg):
    """Seeded Gaussian mixture (centres N(0,1), sigma per dim), L2-normalised, and queries =
    random database rows + N(0, qsigma) noise, renormalised."""
    rng = np.random.default_rng(cfg["seed"])
    n, d = cfg["n"], cfg["d"]
    cent = rng.standard_normal((cfg["centres"], d), dtype=np.float32)
    X = np.empty((n, d), np.float32)
    step = 1 << 17
    for a in range(0, n, step):
        b = min(n, a + step)
        X[a:b] = cent[rng.integers(0, cfg["centres"], b - a)]
        X[a:b] += np.float32(cfg["sigma"]) * rng.standard_normal((b - a, d), dtype=np.float32)
        X[a:b] /= np.linalg.norm(X[a:b], axis=1, keepdims=True)
    src = rng.integers(0, n, cfg["nq"])
    Q = X[src] + np.float32(cfg["qsigma"]) * rng.standard_normal((cfg["nq"], d), dtype=np.float32)
    Q /= np.linalg.norm(Q, axis=1, keepdims=True)
    return X, np.ascontiguousarray(Q, np.float32)


def make_data_device(cfg, dev):
    """Config 4 / 5 data on the device (rbq_gen_mixture / rbq_gen_queries: seeded Philox mixture,
    per-dim scale sqrt(1/(1+d/64)) when anisotropic, L2-normalised; queries = database rows +
    N(0, qsigma) noise, renormalised)."""
    import torch

    from neurosamble_b200 import _lib
    from neurosamble_b200.index import _ptr, _stream_ptr
    n, d, nq = cfg["n"], cfg["d"], cfg["nq"]
    X = torch.empty((n, d), dtype=torch.float32, device=dev)
    Q = torch.empty((nq, d), dtype=torch.float32, device=dev)
    st = _stream_ptr(dev.index)
    _lib.call("rbq_gen_mixture", _ptr(X), n, d, cfg["centres"], cfg["sigma"], cfg["aniso"], 1, cfg["seed"], st)
    _lib.call("rbq_gen_queries", _ptr(X), n, d, _ptr(Q), nq, cfg["qsigma"], 1, cfg["seed"] + 1, None, st)
    torch.cuda.synchronize(dev)
    return X, Q


def make_data_reads(cfg, dev, rank=0, world=1):
    """Config 3: embeddings of simulated reads (bench_reads.make_read_embeddings); each rank
    encodes its share of the read batches and a sum all-reduce assembles the whole set (rows
    of other ranks' batches are zero).  The queries are the reads themselves."""
    import torch

    import bench_reads
    X, _, _ = bench_reads.make_read_embeddings(cfg["n"], cfg["read_len"], cfg["genome_len"], cfg["seed"], dev,
                                               d=cfg["d"], rank=rank, world=world, log=log)
    if world > 1:
        import torch.distributed as tdist
        tdist.all_reduce(X, op=tdist.ReduceOp.SUM)
    torch.cuda.synchronize(dev)
    return X, X[:cfg["nq"]]


def exact_knn_device(Xd, Qs, k, rows=1 << 20, qblock=1000):
    """Exact k nearest rows (fp32 |x|^2 - 2 q.x, running top-k over row chunks) of the sample Qs."""
    import torch
    out = []
    for qa in range(0, Qs.shape[0], qblock):
        q = Qs[qa:qa + qblock]
        bd = bi = None
        for a in range(0, Xd.shape[0], rows):
            xb = Xd[a:a + rows]
            s = (xb * xb).sum(1)[None, :] - 2.0 * (q @ xb.T)
            d_, i_ = torch.topk(s, min(k, s.shape[1]), dim=1, largest=False)
            i_ = i_ + a
            if bd is not None:
                d_, j = torch.topk(torch.cat([bd, d_], 1), k, dim=1, largest=False)
                i_ = torch.gather(torch.cat([bi, i_], 1), 1, j)
            bd, bi = d_, i_
            del s
        out.append(bi.cpu())
    return torch.cat(out).numpy()


def measured_peak():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
           0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
           0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled every 10 ms during the timed region,
    read through NVML (read-only queries; nothing is set).  Only rank 0 samples (its own GPU):
    eight processes polling NVML at once slowed every rank's kernel launches."""

    def __init__(self, gpu_index: int, active: bool = True):
        self.gpu = gpu_index
        self.active = active
        self.samples = []
        self.stop = threading.Event()
        self.t = None

    def _handle(self, nv):
        import torch
        try:
            return nv.nvmlDeviceGetHandleByUUID("GPU-" + str(torch.cuda.get_device_properties(self.gpu).uuid))
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(self.gpu)

    def __enter__(self):
        if not self.active:
            return self
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            mx = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))

            def run():
                while not self.stop.is_set():
                    try:
                        self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), mx,
                                             int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))))
                    except Exception:
                        pass
                    self.stop.wait(0.010)

            self.t = threading.Thread(target=run, daemon=True)
            self.t.start()
        except Exception:
            self.t = None
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.t:
            self.t.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(s[0] for s in self.samples)
        mask = 0
        for s in self.samples:
            mask |= s[2]
        names = [v for k, v in REASONS.items() if mask & k and k != 0x1]
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": max(s[1] for s in self.samples), "reasons": names,
                "samples": len(self.samples)}


# --------------------------------------------------------------------------------------
# reference arm: the CPU restatement of the reference search, all host cores
# --------------------------------------------------------------------------------------
def blas_assign(A, C):
    """Nearest centre by a BLAS argmin of |c|^2 - 2 a.c (the CPU arm's build; not timed)."""
    out = np.empty(A.shape[0], np.uint32)
    cn = (C * C).sum(1)[None, :]
    for a in range(0, A.shape[0], 65536):
        out[a:a + 65536] = np.argmin(cn - 2.0 * A[a:a + 65536] @ C.T, axis=1)
    return out


def kmeans_numpy(X, k, iters, per_list, seed, kind="balanced"):
    """Training for the CPU arm (not timed): the strided sample the library trains on, then the
    same trainer as our arm (balanced k-means restated in the oracle, or Lloyd), BLAS E steps."""
    n = X.shape[0]
    m = min(n, per_list * k)
    S = X[(np.arange(m, dtype=np.int64) * n) // m]
    if kind == "balanced":
        from oracle import oracle as O
        return O.kmeans_balanced(S, k, iters, assign_fn=blas_assign)
    C = S[(np.arange(k, dtype=np.int64) * m) // k].copy()

    for _ in range(iters):
        lab = blas_assign(S, C)
        sums = np.zeros((k, X.shape[1]), np.float64)
        np.add.at(sums, lab, S)
        cnt = np.bincount(lab, minlength=k)
        nz = cnt > 0
        C[nz] = (sums[nz] / cnt[nz, None]).astype(np.float32)
    return C


def list_scan_used(cfg, world=1, R=0):
    """Whether the library's search of the whole batch takes the list scan (its auto rule:
    popcount modes, padded dim <= 768, nq * nprobe >= 64 * nlist, n >= max(R, k) * nlist; scan_kind
    1 / 2 force the tile /
    list scan; the sharded search follows the same rule).  The CPU oracle is told the same, so
    that its sample answers like the full batch."""
    dp = (cfg["d"] + 31) // 32 * 32
    kind = cfg.get("scan_kind", 0)
    able = cfg["query_bits"] in (4, 8) and dp <= 768
    auto = (cfg["nq"] * cfg["nprobe"] >= 64 * cfg["nlist"]
            and cfg["n"] >= max(R, cfg["k"]) * cfg["nlist"])
    return able and (kind == 2 or (kind == 0 and auto))


def cpu_search_timed(O, oix, Q, cfg, R, budget_s=20.0, scan_kind=None):
    """Time the oracle search on a bounded query sample sized to ~budget_s of CPU work.  scan_kind
    None: the scan the library's search of the batch takes (for parity); 1: the tile scan, the
    reference's own algorithm (a per-query scan with a running pruning threshold)."""
    sk = scan_kind if scan_kind is not None else (2 if list_scan_used(cfg, 1, R) else 1)
    probe = min(len(Q), 200)
    t0 = time.perf_counter()
    O.search(oix, Q[:probe], cfg["k"], cfg["nprobe"], R, query_bits=cfg["query_bits"], scan_kind=sk)
    per_q = (time.perf_counter() - t0) / probe
    n = int(min(len(Q), max(probe, budget_s / max(per_q, 1e-9))))
    t0 = time.perf_counter()
    d, i = O.search(oix, Q[:n], cfg["k"], cfg["nprobe"], R, query_bits=cfg["query_bits"], scan_kind=sk)
    dt = time.perf_counter() - t0
    return n / dt, n, dt, (d, i)


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle import oracle as O
    if cfg.get("generator") == "reads":  # the inputs come from the signal encoder (GPU); not timed
        import torch
        Xd, _ = make_data_reads(cfg, torch.device("cuda:0"))
        X = Xd.cpu().numpy()
        Q = X[:cfg["nq"]]
        del Xd
    else:
        X, Q = make_data(cfg)
    dp = O.pad_dim(cfg["d"])
    P = O.make_rotation(dp, 7)
    t4 = O.query_scale(dp, 7)
    t = time.perf_counter()
    C = kmeans_numpy(X, cfg["nlist"], 20, 256, cfg["seed"], args.kmeans)
    cn = (C * C).sum(1)[None, :]
    lab = np.concatenate([np.argmin(cn - 2.0 * X[a:a + 65536] @ C.T, axis=1)
                          for a in range(0, cfg["n"], 65536)]).astype(np.uint32)
    bpd = cfg.get("bits_per_dim", 1)
    oix = O.build(X, C, lab, P, t4, bits_per_dim=bpd, tex=O.ex_scale(dp, 7, bpd - 1, t4) if bpd > 1 else None)
    oix.t8 = O.query_scale(dp, 7, 7)
    log(f"[reference] build {time.perf_counter() - t:.1f}s, threads={O.threads()}")
    # the same recall rule as our arm: the smallest rerank depth on the ladder whose recall@k
    # reaches the target, measured here on a 500-query sample against exact neighbours
    recalls = {}
    if args.rerank:
        R = args.rerank
    else:
        ns = min(500, len(Q))
        xn = (X * X).sum(1)
        gt = np.concatenate([np.argpartition(xn[None, :] - 2.0 * (Q[a:a + 100] @ X.T), cfg["k"], axis=1)[:, :cfg["k"]]
                             for a in range(0, ns, 100)])
        R = rerank_ladder(cfg)[-1]
        for cand in rerank_ladder(cfg):
            _, ids = O.search(oix, Q[:ns], cfg["k"], cfg["nprobe"], cand, query_bits=cfg["query_bits"],
                              scan_kind=1)
            recalls[cand] = O.recall(ids, gt)
            if recalls[cand] >= RECALL_TARGET:
                R = cand
                break
        log(f"[reference] recall@{cfg['k']} on {ns} queries by rerank depth: {recalls}; using R={R}")
    steps = []
    n_sample = None
    for s in range(args.warmup + args.steps):
        qps, n, dt, _ = cpu_search_timed(O, oix, Q, cfg, R, budget_s=max(2.0, 60.0 / (args.steps + args.warmup)),
                                         scan_kind=1)
        if s >= args.warmup:
            steps.append(qps)
            n_sample = n
    value = float(np.mean(steps))
    line = {"impl": "reference", "metric": metric_name(cfg), "value": round(value, 2), "unit": "queries/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1000.0 * cfg["nq"] / value, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32+u32",
            "data": data_label(cfg),
            "config": dict(workload(cfg, R, args.kmeans), recall_by_rerank_sample=recalls),
            "cpu_baseline": {"value": round(value, 2), "unit": "queries/s", "cores": O.threads(), "kind": "port",
                             "sample": f"{n_sample} of {cfg['nq']} queries per step, same index and parameters",
                             "timed_scan": "tile (the reference's per-query pruned scan)"},
            "e2e": {"value": round(value, 2), "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def data_label(cfg):
    if cfg.get("generator") == "reads":
        return "synthetic (simulated reads embedded by a seeded random-init signal encoder, BASELINE config 3)"
    return f"synthetic (seeded Gaussian mixture, BASELINE config {cfg['config']})"


def _count(n):
    return f"{n // 1_000_000}M" if n % 1_000_000 == 0 else str(n)


SEARCH_MODES = {4: "QUANT4", 8: "QUANT8", 16: "LUT16", 32: "LUT32"}


def _codes(cfg):
    b = cfg.get("bits_per_dim", 1)
    return "1-bit codes" if b == 1 else f"{b}-bit ExRaBitQ codes"


def metric_name(cfg):
    return (f"queries/sec @ recall@{cfg['k']}>=0.95, {_count(cfg['n'])} x {cfg['d']} IVF-RaBitQ "
            f"(nlist {cfg['nlist']}, nprobe {cfg['nprobe']}, k {cfg['k']})")


def workload(cfg, R, kmeans):
    if cfg.get("generator") == "reads":
        return {"workload": (f"BASELINE config 3: read-overlap retrieval, {cfg['n']} simulated reads of "
                             f"{cfg['read_len']} bp from a seeded {cfg['genome_len'] // 1_000_000} Mbp genome (50% "
                             "reverse-complemented, 8% errors 4:2:2 sub:ins:del), synthetic 6-mer pore-model signal, "
                             "2000/1000 windows, seeded random-init signal encoder (d 256) under fp16 autocast, "
                             "mean-pooled per read, L2-normalised, fp16 -> fp32; the read set queried against itself; "
                             f"IVF-RaBitQ {_codes(cfg)}, {cfg.get('query_bits', 4)}-bit queries; data generated on the "
                             "device"),
                "n": cfg["n"], "dim": cfg["d"], "nlist": cfg["nlist"], "nprobe": cfg["nprobe"], "k": cfg["k"],
                "rerank": R, "query_batch": cfg["nq"], "l2": "flushed before every step (256 MB write)",
                "kmeans": kmeans, "search_mode": SEARCH_MODES[cfg.get("query_bits", 4)]}
    return {"workload": (f"BASELINE config {cfg['config']}: {_count(cfg['n'])} x {cfg['d']} f32, "
                         f"{cfg['centres']}-centre {'anisotropic ' if cfg['aniso'] else ''}mixture sigma "
                         f"{cfg['sigma']}, L2-normalised; {cfg['nq']} perturbed-row queries; IVF-RaBitQ "
                         f"{_codes(cfg)}, {cfg.get('query_bits', 4)}-bit queries"
                         + ("; data generated on the device" if cfg["device_data"] else "")),
            "n": cfg["n"], "dim": cfg["d"], "nlist": cfg["nlist"], "nprobe": cfg["nprobe"], "k": cfg["k"],
            "rerank": R, "query_batch": cfg["nq"], "l2": "flushed before every step (256 MB write)",
            "kmeans": kmeans, "search_mode": SEARCH_MODES[cfg.get("query_bits", 4)]}


# --------------------------------------------------------------------------------------
# our arm
# --------------------------------------------------------------------------------------
def run_ours(args, cfg):
    import ctypes

    import torch
    import torch.distributed as tdist

    from neurosamble_b200 import IndexIVFRaBitQ, _lib
    from neurosamble_b200.index import _ptr, _stream_ptr

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        log(f"[rank {rank}] NCCL_DEBUG={os.environ.get('NCCL_DEBUG')!r} NCCL_DEBUG_FILE={os.environ.get('NCCL_DEBUG_FILE')!r}")
    if world > 1 and os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
        # NCCL's communicator set-up lines (ranks, devices, NVLS) go to stderr, so stdout carries
        # only the JSON line while the log still shows every rank joining
        os.environ.update(NCCL_DEBUG="INFO", NCCL_DEBUG_SUBSYS="INIT", NCCL_DEBUG_FILE="/dev/stderr")
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    group = None
    if world > 1:
        from datetime import timedelta
        tdist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    t = time.perf_counter()
    if cfg.get("generator") == "reads":
        Xd, Qd = make_data_reads(cfg, dev, rank, world)
        X = Xd.cpu().numpy()
        Q = X[:cfg["nq"]]
    elif cfg["device_data"]:
        X = None
        Xd, Qd = make_data_device(cfg, dev)
        Q = Qd.cpu().numpy()
    else:
        X, Q = make_data(cfg)
        Xd = torch.from_numpy(X).to(dev)
        Qd = torch.from_numpy(Q).to(dev)
    log(f"[rank {rank}] data {time.perf_counter() - t:.1f}s")
    t = time.perf_counter()
    if world > 1:
        from neurosamble_b200.sharded import ShardedIndexIVFRaBitQ
        index = ShardedIndexIVFRaBitQ(cfg["d"], cfg["nlist"], seed=7, device=local, kmeans=args.kmeans,
                                      bits_per_dim=cfg.get("bits_per_dim", 1))
        local_ix = index.local
    else:
        index = IndexIVFRaBitQ(cfg["d"], cfg["nlist"], seed=7, device=local, kmeans=args.kmeans,
                               bits_per_dim=cfg.get("bits_per_dim", 1))
        local_ix = index
    index.train(Xd)
    index.add(Xd)
    torch.cuda.synchronize()
    log(f"[rank {rank}] build {time.perf_counter() - t:.1f}s, local vectors {local_ix.info().n_local}")
    index.nprobe = cfg["nprobe"]
    index.prune = True
    index.query_bits = cfg["query_bits"]
    index.scan_kind = args.scan_kind
    if world == 1:
        index.seeded = args.seeded

    # ---- recall at the config's rerank depth; raise R along the ladder until recall >= target
    # (exact neighbours of the first gt_sample queries: all of config 2's, 1,000 at configs 4 / 5)
    gt = None
    ns = min(cfg["gt_sample"], cfg["nq"])
    if rank == 0:
        t = time.perf_counter()
        gt = exact_knn_device(Xd, Qd[:ns], cfg["k"])
        log(f"[rank 0] exact neighbours of {ns} queries {time.perf_counter() - t:.1f}s")
    del Xd
    torch.cuda.empty_cache()

    def recall_of(ids):
        hit = sum(len(set(a.tolist()) & set(b.tolist())) for a, b in zip(ids[:ns], gt))
        return hit / gt.size

    R = args.rerank or cfg["rerank"]
    recalls = {}
    if args.rerank:
        ladder = [R]
    elif cfg["config"] == 2:
        ladder = list(rerank_ladder(cfg))
    else:
        ladder = [min(4096, int(R * f)) for f in (1, 1.5, 2, 3, 4)]
    for cand in ladder:
        index.k_rerank = cand
        d, i = index.search(Qd, cfg["k"])
        ok = torch.zeros(1, dtype=torch.int32, device=dev)
        if rank == 0:
            recalls[cand] = round(recall_of(i.cpu().numpy()), 5)
            ok[0] = int(recalls[cand] >= RECALL_TARGET)
        if world > 1:
            tdist.broadcast(ok, src=0)
        R = cand
        if ok.item():
            break
    index.k_rerank = R
    log(f"[rank {rank}] recall@{cfg['k']} by rerank depth: {recalls}; using R={R}")

    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    k = cfg["k"]
    nq = cfg["nq"]

    def barrier():
        if world > 1:
            tdist.barrier()
        torch.cuda.synchronize(dev)

    last = {}

    def step_device():
        d, i = index.search(Qd, k)
        last["r"] = (d, i)
        return d, i

    # ---- value: device-resident queries
    for _ in range(args.warmup):
        flush.zero_()
        step_device()
    barrier()
    launches0 = _lib.lib().rbq_kernel_launches()
    torch.cuda.nvtx.range_push("timed")
    # Each step's events bracket its search only, not the L2 flush before it.  One GPU: steps are
    # queued back to back (the host runs ahead, as a serving loop does).  Several: the ranks
    # enter every step together through a barrier (which also drains the GPU), because queued
    # steps let the ranks drift and a step's collectives then wait on the previous step's
    # stragglers, which measured 20-50 % slower and varied from run to run.
    evs = []
    with ClockSampler(local, active=rank == 0) as clk:
        for _ in range(args.steps):
            flush.zero_()
            if world > 1:
                tdist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step_device()
            e1.record(stream)
            evs.append((e0, e1))
        torch.cuda.synchronize(dev)
    torch.cuda.nvtx.range_pop()
    barrier()
    times = [a.elapsed_time(b) for a, b in evs]
    launches = _lib.lib().rbq_kernel_launches() - launches0
    ms = float(np.mean(times))
    if world > 1:
        t_max = torch.tensor([ms], device=dev)
        tdist.all_reduce(t_max, op=tdist.ReduceOp.MAX)
        ms = float(t_max.item())
    value = nq / (ms / 1000.0)

    # ---- e2e: host buffers through the C ABI (queries H2D, results D2H inside the timed call)
    Qh = torch.from_numpy(Q).pin_memory()
    dh = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    ih = torch.empty((nq, k), dtype=torch.int64).pin_memory()
    sp = local_ix.search_params(k)
    e2e_times = []

    def step_host():
        if world == 1:
            _lib.call("rbq_search_host", local_ix.handle, ctypes.byref(sp), ctypes.c_void_p(Qh.data_ptr()), nq,
                      ctypes.c_void_p(dh.data_ptr()), ctypes.c_void_p(ih.data_ptr()), _stream_ptr(local))
        else:
            qd = Qh.to(dev, non_blocking=True)
            d, i = index.search(qd, k)
            dh.copy_(d, non_blocking=True)
            ih.copy_(i, non_blocking=True)
            torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        flush.zero_()
        torch.cuda.synchronize(dev)
        step_host()
    barrier()
    for _ in range(args.steps):
        flush.zero_()
        torch.cuda.synchronize(dev)
        if world > 1:
            tdist.barrier()
        t0 = time.perf_counter()
        step_host()
        e2e_times.append(time.perf_counter() - t0)
    e2e_s = float(np.median(e2e_times))  # host timers: the median resists scheduler noise
    if world > 1:
        t_max = torch.tensor([e2e_s], device=dev)
        tdist.all_reduce(t_max, op=tdist.ReduceOp.MAX)
        e2e_s = float(t_max.item())
    e2e = nq / e2e_s

    # ---- N > 1: one more search with CUDA events at its stage boundaries (front end, the three
    # collectives, scan, rerank, merge); rank 0's milliseconds and the max over ranks
    stages_ms = None
    if world > 1:
        tdist.barrier()
        tm = {}
        index.search(Qd, k, timings=tm)
        names = list(tm)
        vals = torch.tensor([tm[n] for n in names], dtype=torch.float64, device=dev)
        vmax = vals.clone()
        tdist.all_reduce(vmax, op=tdist.ReduceOp.MAX)
        stages_ms = {"rank0": {n: round(float(v), 4) for n, v in zip(names, vals.tolist())},
                     "max_over_ranks": {n: round(float(v), 4) for n, v in zip(names, vmax.tolist())}}

    # ---- roofline of the dominant kernel (the list scan), live CUDA events on its stream
    seeded = (world > 1 or args.seeded == 1) and cfg["query_bits"] < 16  # LUT modes: one pass, no seed
    lists = list_scan_used(cfg, world, R)
    roof, roof_rr = scan_roofline(local_ix, Qd, cfg, R, flush, args.steps, dev, seeded, lists)
    scan_share = round(roof["launch_ms"] / ms, 3)

    # ---- config 2's batch sweep (B = 1, 64, 1024): device-resident queries, same index
    sweep = sweep_graph = None
    if world == 1 and not args.no_sweep and cfg["config"] == 2:
        def sweep_once():
            out = {}
            for B in (1, 64, 1024):
                qb = Qd[:B]
                reps = max(3, min(200, 20000 // B))
                for _ in range(3):  # warm-up (captures the graph in graph mode)
                    index.search(qb, k)
                torch.cuda.synchronize(dev)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(reps):
                    index.search(qb, k)
                e1.record(stream)
                e1.synchronize()
                ms_b = e0.elapsed_time(e1) / reps
                out[str(B)] = {"queries_per_s": round(B / (ms_b / 1000.0), 1), "ms_per_batch": round(ms_b, 4)}
            return out
        sweep = sweep_once()
        sweep["10000"] = {"queries_per_s": round(value, 1), "ms_per_batch": round(ms, 4)}
        index.use_graph = True  # the same searches replayed from captured CUDA graphs
        sweep_graph = sweep_once()
        index.use_graph = False

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and X is not None:
        gd, gi = last["r"]
        cpu = cpu_baseline(local_ix, X, Q, cfg, R, (gd.cpu().numpy(), gi.cpu().numpy()))

    if world > 1:
        tdist.barrier()
    if rank == 0:
        line = {"metric": metric_name(cfg), "value": round(value, 2), "unit": "queries/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None,
                "dtype": ("s8 query codes x u8 code bits (tcgen05 i8) + f32" if lists
                          else "u32 codes x 4-bit planes (popc) + f32"),
                "data": data_label(cfg),
                "config": dict(workload(cfg, R, args.kmeans),
                               parallelism=(f"lists sharded over {world} GPUs (balanced by size^2)" if world > 1
                                            else "1 GPU"),
                               scan=("list scan (fixed thresholds, tensor-core list GEMM)" if lists
                                     else "tile scan"),
                               recall_by_rerank=recalls, **{f"recall_at_{k}": recalls.get(R)}),
                "clocks": clk.summary(),
                "e2e": {"value": round(e2e, 2), "unit": "queries/s", "h2d_bytes_per_step": nq * cfg["d"] * 4,
                        "d2h_bytes_per_step": nq * k * 12},
                "gpu_launches": int(launches),
                "roofline": roof, "roofline_rerank": roof_rr, "scan_share_of_step": scan_share,
                "batch_sweep": sweep, "batch_sweep_graph": sweep_graph,
                "stages_ms": stages_ms,
                "cpu_baseline": cpu}
        print(json.dumps(line), flush=True)
    if world > 1:
        tdist.destroy_process_group()
    return 0


def scan_roofline(ix, Qd, cfg, R_search, flush, steps, dev, seeded, lists=False):
    """Time the scan and rbq_rerank alone on the batch, as the search runs them (lists: the bound
    seeds and the tensor-core list scan; seeded: the nearest probe, then the others from the
    threshold it gives, all-reduced across shards; else one tile scan);
    algorithmic bytes from the actual probed list sizes: sum n_l (D/8 + 12) for the scan,
    (4D + 8) per candidate the rerank holds.  Without a rerank (R_search 0) the scan keeps k
    candidates and there is no rerank line."""
    R = max(R_search, cfg["k"])
    import ctypes

    import torch

    from neurosamble_b200 import _lib
    from neurosamble_b200.index import _ptr, _stream_ptr

    nq, d, P = Qd.shape[0], cfg["d"], cfg["nprobe"]
    info = ix.info()
    dp = info.padded_dim
    h, st = ix.handle, _stream_ptr(dev.index)
    qr = torch.empty((nq, dp), dtype=torch.float32, device=dev)
    qb = cfg["query_bits"]
    lut = qb in (16, 32)  # LUT16 / LUT32 scan from 4-bit planes' k1 and tables of the float query
    planes = torch.empty((nq, 8 if qb == 8 else 4, dp // 32), dtype=torch.int32, device=dev)
    delta = torch.empty(nq, dtype=torch.float32, device=dev)
    k1 = torch.empty(nq, dtype=torch.float32, device=dev)
    probes = torch.empty((nq, P), dtype=torch.int32, device=dev)
    g = torch.empty((nq, P), dtype=torch.float32, device=dev)
    _lib.call("rbq_rotate", h, _ptr(Qd), nq, _ptr(qr), st)
    _lib.call("rbq_coarse", h, _ptr(qr), nq, P, 0, _ptr(probes), _ptr(g), st)
    _lib.call("rbq_query_prep", h, _ptr(qr), nq, _ptr(planes), _ptr(delta), _ptr(k1), qb, st)
    torch.cuda.synchronize(dev)
    sizes = np.diff(ix.list_offsets())
    pr = probes.cpu().numpy()
    owned = ix.list_owners()[pr] == info.shard_rank
    vec = int(sizes[pr][owned].sum())
    scan_bytes = vec * (d // 8 + (8 if lut else 12))  # the table estimate reads no error factor
    stream = torch.cuda.current_stream(dev)
    stats = torch.zeros(2, dtype=torch.int64, device=dev)

    def timed(fn):
        ts = []
        for it in range(3 + steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            if it >= 3:
                ts.append(e0.elapsed_time(e1))
        return float(np.mean(ts))

    def scan(pp, gg, npr, tau, init, ids_t, dist_t, stats_t):
        _lib.call("rbq_scan", h, _ptr(qr), _ptr(planes), _ptr(delta), _ptr(k1), nq, _ptr(pp), _ptr(gg), npr,
                  pp.stride(0), _ptr(tau) if tau is not None else None, _ptr(init[0]) if init else None,
                  _ptr(init[1]) if init else None, R, 1, 1, 0, _ptr(ids_t), _ptr(dist_t),
                  _ptr(stats_t) if stats_t is not None else None, qb, st)

    ids = torch.empty((nq, R), dtype=torch.int64, device=dev)
    dist = torch.empty((nq, R), dtype=torch.float32, device=dev)
    if lists:  # the search's list scan, stage by stage: bound seeds over the leading probed lists,
        # the tile scan of the nearest probe from them, the nearest list's R-th distance as the
        # fixed threshold of the list scan of the other probes, the merge of both
        tau_l = torch.empty(nq, dtype=torch.float32, device=dev)
        dd = torch.empty((2, nq, R), dtype=torch.float32, device=dev)
        ii = torch.empty((2, nq, R), dtype=torch.int64, device=dev)
        pa, ga = probes[:, :1], g[:, :1]  # strided column views, row stride P
        pb, gb = probes[:, 1:], g[:, 1:]

        def run_lists(stats_t):
            sp_ = _ptr(stats_t) if stats_t is not None else None
            # sharded: the seed on the nearest probe's owner only, then the minimum over the ranks
            _lib.call("rbq_bound_seed_owned" if info.shard_count > 1 else "rbq_bound_seed", h, _ptr(qr), _ptr(planes),
                      _ptr(delta), _ptr(k1), nq, _ptr(probes), _ptr(g), P, P, R, 0, _ptr(tau_l), qb, st)
            if info.shard_count > 1:
                import torch.distributed as tdist
                tdist.all_reduce(tau_l, op=tdist.ReduceOp.MIN)
            _lib.call("rbq_scan", h, _ptr(qr), _ptr(planes), _ptr(delta), _ptr(k1), nq, _ptr(pa), _ptr(ga), 1, P,
                      _ptr(tau_l), None, None, R, 1, 1, 0, _ptr(ii[0]), _ptr(dd[0]), sp_, qb, st)
            if P == 1:
                ids.copy_(ii[0])
                dist.copy_(dd[0])
                return
            tau1 = torch.where(ii[0][:, R - 1] >= 0, torch.minimum(tau_l, dd[0][:, R - 1]), tau_l).contiguous()
            if info.shard_count > 1:
                import torch.distributed as tdist
                tdist.all_reduce(tau1, op=tdist.ReduceOp.MIN)
            _lib.call("rbq_scan_lists", h, _ptr(qr), _ptr(planes), _ptr(delta), _ptr(k1), nq, _ptr(pb), _ptr(gb),
                      P - 1, P, _ptr(tau1), R, _ptr(ii[1]), _ptr(dd[1]), sp_, qb, st)
            _lib.call("rbq_merge_results", _ptr(dd), _ptr(ii), 2, nq, R, _ptr(dist), _ptr(ids), st)

        run_lists(stats)
        scan_ms = timed(lambda: run_lists(None))
    elif seeded:  # the search's two phases: the nearest probe, then the rest from the shared seed
        ia = torch.empty((nq, R), dtype=torch.int64, device=dev)
        da = torch.empty((nq, R), dtype=torch.float32, device=dev)
        pa, ga = probes[:, :1], g[:, :1]  # strided column views, row stride P
        pb, gb = probes[:, 1:], g[:, 1:]
        scan(pa, ga, 1, None, None, ia, da, stats)
        tau = da[:, R - 1].contiguous()
        if info.shard_count > 1:
            import torch.distributed as tdist
            tdist.all_reduce(tau, op=tdist.ReduceOp.MIN)
        scan(pb, gb, P - 1, tau, (ia, da), ids, dist, stats)

        def run_scan():
            scan(pa, ga, 1, None, None, ia, da, None)
            scan(pb, gb, P - 1, tau, (ia, da), ids, dist, None)

        scan_ms = timed(run_scan)
    else:
        scan(probes, g, P, None, None, ids, dist, stats)
        scan_ms = timed(lambda: scan(probes, g, P, None, None, ids, dist, None))
    scanned, admitted = (int(v) for v in stats.cpu().tolist())
    od = torch.empty((nq, cfg["k"]), dtype=torch.float32, device=dev)
    oi = torch.empty((nq, cfg["k"]), dtype=torch.int64, device=dev)
    rr_ms = timed(lambda: _lib.call("rbq_rerank", h, _ptr(Qd), nq, _ptr(ids), R, cfg["k"], _ptr(od), _ptr(oi), st)) \
        if R_search > 0 else None
    n_valid = int((ids >= 0).sum().item())
    rr_bytes = n_valid * (4 * d + 8)
    peak, kind = measured_peak()
    # DRAM traffic cannot be read inside a plain run: it comes from a stored ncu capture of the
    # same kernel and workload (profiles/scan_traffic.json), and the line says so
    traffic, traffic_src = None, None
    tname = "list_scan_traffic.json" if lists else "scan_traffic.json"
    tf = os.path.join(HERE, "profiles", tname)
    if os.path.exists(tf):
        try:
            with open(tf) as f:
                tj = json.load(f)
            if tj.get("config", 2) == cfg.get("config", 2):
                traffic = tj.get("bytes_per_launch_scaled_to_bench")
                traffic_src = f"stored ncu capture (profiles/{tname}), not measured in this run"
        except Exception:
            traffic = None
    ach = scan_bytes / (scan_ms / 1000.0) / 1e9
    roof = {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
            "traffic": traffic, "traffic_source": traffic_src, "peak_kind": kind,
            "kernel": ("rbq list scan: bound seeds, tile scan of the nearest probe, tcgen05 kind::i8 list GEMM + "
                       "admission, exact pass per query, merge"
                       if lists else "rbq scan_kernel (+ key->id epilogue)"
                       + (", 2 launches: seed list + rest" if seeded else "")),
            "accounting": ("algorithmic bytes per query summed over the batch; the list scan reads each list once "
                           "for up to 128 of its queries, so the fraction can exceed 1" if lists else
                           "algorithmic bytes per query summed over the batch"),
            "algorithmic_bytes_per_launch": scan_bytes, "probed_vectors_per_launch": vec,
            "launch_ms": round(scan_ms, 4), "prune_admitted_fraction": round(admitted / max(1, scanned), 4)}
    if rr_ms is None:
        return roof, None
    ach_r = rr_bytes / (rr_ms / 1000.0) / 1e9
    roof_rr = {"bound": "hbm", "achieved": round(ach_r, 1), "peak": peak, "unit": "GB/s",
               "frac": round(ach_r / peak, 4), "kernel": "rbq rerank_kernel (+ id->key prologue)",
               "algorithmic_bytes_per_launch": rr_bytes, "launch_ms": round(rr_ms, 4)}
    return roof, roof_rr


def cpu_baseline(ix, X, Q, cfg, R, gpu_result=None):
    """The oracle (the CPU restatement of the reference search), all host cores, on a bounded
    sample of the same batch against the same index.  With gpu_result = (dist, ids) of the
    timed GPU search of the whole batch, the oracle's answers for the sample are compared with
    the GPU's for the same queries (the line's `parity` object)."""
    from oracle import oracle as O
    ex = ix.export_lists()
    C, Cr = ix.centroids()
    info = ix.info()
    n = X.shape[0]
    # the oracle's index arrays are the GPU index's own (same layout, same bytes)
    oix = O.OracleIndex(cfg["d"], info.padded_dim, cfg["nlist"], ex["list_off"], ex["ids"], ex["codes"], ex["fadd"],
                        ex["frescale"], ex["ferr"], Cr, ix.rotation(), ix.query_scale, X)
    oix.t8 = O.query_scale(info.padded_dim, int(info.seed), 7)
    if info.bits_per_dim > 1:
        oix.set_ex(ex["ex_bits"], ex["ex_codes"], ex["fexadd"], ex["fexr"], ex["ex_scale"])
    # timed: the reference's algorithm (the tile scan); parity: the scan the GPU search took
    qps, n_s, dt, (od, oi) = cpu_search_timed(O, oix, Q, cfg, R, budget_s=15.0, scan_kind=1)
    out = {"value": round(qps, 2), "unit": "queries/s", "cores": O.threads(), "kind": "port",
           "sample": f"{n_s} of {cfg['nq']} queries ({dt:.1f}s), same index bytes and parameters",
           "timed_scan": "tile (the reference's per-query pruned scan)"}
    if gpu_result is not None:
        lists = list_scan_used(cfg, 1, R)
        if lists:
            _, n_p, _, (od, oi) = cpu_search_timed(O, oix, Q, cfg, R, budget_s=15.0)
        else:
            n_p = n_s
        out["parity"] = parity_of(gpu_result[0][:n_p], gpu_result[1][:n_p], od, oi)
        out["parity"]["scan"] = "list" if lists else "tile"
    return out


def parity_of(gd, gi, od, oi, rel_tol=1e-4):
    """GPU result against the oracle's for the same queries on the same index bytes: ids equal,
    distance bits equal, the largest relative distance error over finite entries, and the ids
    that differ outside distance ties within rel_tol (the north star's tie rule)."""
    gd = np.asarray(gd, np.float32)
    od = np.asarray(od, np.float32)
    gi = np.asarray(gi)
    oi = np.asarray(oi)
    fin = np.isfinite(gd) & np.isfinite(od)
    rel = np.abs(gd[fin].astype(np.float64) - od[fin]) / np.maximum(np.abs(od[fin].astype(np.float64)), 1e-30)
    diff_rows = np.nonzero((gi != oi).any(axis=1))[0]
    untied = 0
    for r in diff_rows:  # a differing id is a tie if its distance equals the other side's within rel_tol
        for j in np.nonzero(gi[r] != oi[r])[0]:
            if abs(float(gd[r, j]) - float(od[r, j])) > rel_tol * max(abs(float(od[r, j])), 1e-30):
                untied += 1
    return {"n": int(gi.shape[0]), "k": int(gi.shape[1]), "ids_equal": bool(np.array_equal(gi, oi)),
            "dist_bits_equal": bool(np.array_equal(gd.view(np.uint32), od.view(np.uint32))),
            "max_rel_err": float(rel.max()) if rel.size else 0.0, "rows_differing": int(diff_rows.size),
            "ids_differing_outside_ties": int(untied), "rel_tol": rel_tol}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--rerank", type=int, default=0, help="fixed rerank depth (0 = smallest meeting recall 0.95)")
    ap.add_argument("--n", type=int, default=0, help="database size override (smoke runs)")
    ap.add_argument("--nq", type=int, default=0, help="query batch override")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="skip the B = 1 / 64 / 1024 sweep")
    ap.add_argument("--kmeans", default="balanced", choices=["balanced", "lloyd"],
                    help="coarse trainer of both arms (balanced: the reference's build algorithm)")
    ap.add_argument("--query-bits", type=int, default=4, choices=sorted(SEARCH_MODES),
                    help="search mode of both arms: 4 (QUANT4, the reference CLI's default), 8 (QUANT8), "
                         "16 (LUT16) or 32 (LUT32)")
    ap.add_argument("--bits", type=int, default=1, choices=range(1, 10),
                    help="code bits per dimension of both arms (1: RaBitQ; 2..9: ExRaBitQ extra bits)")
    ap.add_argument("--scan-kind", type=int, default=0, choices=[0, 1, 2],
                    help="0: the library's choice (the list scan for large batches), 1: the tile scan, 2: the list scan")
    ap.add_argument("--nlist", type=int, default=0,
                    help="list count override (reduced-size cases of a configuration's shape; mixtures keep "
                         "one centre per list)")
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS),
                    help="benchmark configuration (2: the metric's; 3: read overlap; 4 / 5: supplementary, data on "
                         "the device)")
    ap.add_argument("--seeded", type=int, default=-1, choices=[-1, 0, 1],
                    help="1 GPU: two-phase scan seeded by the nearest list (-1: the library's auto rule)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    cfg["query_bits"] = args.query_bits
    cfg["bits_per_dim"] = args.bits
    cfg["scan_kind"] = args.scan_kind
    if args.n:
        cfg["n"] = args.n
    if args.nq:
        cfg["nq"] = args.nq
    if args.nlist:
        if cfg.get("centres") == cfg["nlist"]:
            cfg["centres"] = args.nlist
        cfg["nlist"] = args.nlist
    if args.impl == "reference":
        if cfg["device_data"] and cfg.get("generator") != "reads":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"config {args.config}: the CPU port needs "
                                  "the whole raw store and a CPU-built index on the host; run at config 2"}))
            return 0
        return run_reference(args, cfg)
    return run_ours(args, cfg)


if __name__ == "__main__":
    sys.exit(main())
