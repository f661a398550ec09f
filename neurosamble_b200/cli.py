"""``rabitq_search``-compatible command line over the B200 library.

    python -m neurosamble_b200.cli --emb reads.f16 --n N --d 256 --nlist 2048 --nprobe 48 \\
        --topk 20 --rerank 200 [--index idx.rbq] [--out_nbr neighbors.i64] [--out_dist dists.f32]

Flags, defaults and files follow src/rabitq_gpu/rabitq_search.cu:72-91: the fp16 [N, D]
embeddings are indexed and then searched all-vs-all in batches of ``--batch`` rows, and the
results are appended to ``neighbors.i64`` (int64 [N, topk]) and ``dists.f32`` (float32
[N, topk], squared L2 estimates in ascending order), the files map_full.py:275-279 maps.
``--index`` reuses a saved index when the file exists and saves the built one otherwise.

Additions: ``--encode_dir`` reads the encoder's shard manifest instead of one flat file;
``--rerank R`` re-ranks the top R estimates with exact fp32 distances (0 keeps the reference
behaviour); ``--metric ip`` writes inner products 1 - d/2 of unit vectors (FAISS's IP view,
descending) instead of squared L2; ``--gpus N`` shards the lists over N GPUs of this node by
relaunching the same command as N processes through torch.distributed.run (127.0.0.1, a free
port).  Under torchrun (WORLD_SIZE > 1, one rank per GPU) the lists are sharded over the
ranks and rank 0 writes the files.

``--bits B`` (1..9, as the reference's ``bits_per_dim``): 1-bit RaBitQ codes, or ExRaBitQ codes with
B - 1 extra bits per dimension whose distance ranks the vectors the 1-bit estimate admits;
``--search_mode`` QUANT4 / QUANT8 (popcount
estimator over 4- or 8-bit query codes) or LUT16 / LUT32 (fp16 / fp32 tables of the float query,
the estimate is the candidate distance); ``--strategy
none`` turns the error-bound prune off, ``centroid_reorder`` keeps it on, with this library's
threshold seeds in place of the reference's centroid-distance seed (``--reorder_scale`` is
accepted and has no effect); ``--stream`` / ``--stream_batch`` (the build always streams
rows from the host in batches of ``--stream_batch``); ``--kmeans_iters`` and
``--train_per_cluster`` as in the reference.
"""
from __future__ import annotations

import argparse
import os
import socket
import subprocess
import sys
import time

import numpy as np

# --search_mode -> IndexIVFRaBitQ.query_bits (search_mode, ivf_rabitq.hpp:113-118)
SEARCH_MODES = {"QUANT4": 4, "QUANT8": 8, "LUT16": 16, "LUT32": 32}


def parse_args(argv=None) -> argparse.Namespace:
    ap = argparse.ArgumentParser(prog="neurosamble_b200.cli", description=__doc__.splitlines()[0])
    ap.add_argument("--emb", default="", help="flat fp16 [N, D] embeddings")
    ap.add_argument("--encode_dir", default="", help="directory holding encode_manifest.json")
    ap.add_argument("--out_nbr", default="neighbors.i64")
    ap.add_argument("--out_dist", default="dists.f32")
    ap.add_argument("--index", default="", help="index file to reuse (if present) or save")
    ap.add_argument("--n", type=int, default=0)
    ap.add_argument("--d", type=int, default=384)
    ap.add_argument("--nlist", type=int, default=21185)
    ap.add_argument("--nprobe", type=int, default=384)
    ap.add_argument("--topk", type=int, default=128)
    ap.add_argument("--bits", type=int, default=1)
    ap.add_argument("--batch", type=int, default=16384)
    ap.add_argument("--kmeans_iters", type=int, default=20)
    ap.add_argument("--search_mode", default="QUANT4")
    ap.add_argument("--strategy", default="centroid_reorder", choices=["centroid_reorder", "none"])
    ap.add_argument("--reorder_scale", type=float, default=1.45)
    ap.add_argument("--stream", type=int, default=0)
    ap.add_argument("--stream_batch", type=int, default=200000)
    ap.add_argument("--train_per_cluster", type=int, default=256)
    ap.add_argument("--rerank", type=int, default=0)
    ap.add_argument("--metric", default="l2", choices=["l2", "ip"])
    ap.add_argument("--seed", type=int, default=7, help="rotation / query-scale seed")
    ap.add_argument("--gpus", type=int, default=1, help="GPUs of this node to shard the lists over")
    ap.add_argument("--raw_store", default="device", choices=["device", "host"],
                    help="where the rerank's raw fp32 rows live: HBM, or pinned host memory read over PCIe "
                         "(raw sets larger than the GPU's memory)")
    return ap.parse_args(argv)


def relaunch_cmd(argv, gpus: int, port: int):
    """The torch.distributed.run command that runs this CLI as `gpus` ranks of one node."""
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
            "--master-addr=127.0.0.1", f"--master-port={port}", "-m", "neurosamble_b200.cli", *argv]


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def check_args(a: argparse.Namespace) -> str:
    """'' when the flags are usable, else the message the reference would print."""
    if not a.emb and not a.encode_dir:
        return "need --emb <fp16 file> --n <N> [--d 384] (or --encode_dir <dir>)"
    if a.emb and a.n <= 0:
        return "need --emb <fp16 file> --n <N> [--d 384]"
    if a.gpus < 1:
        return "--gpus must be >= 1"
    if not 1 <= a.bits <= 9:
        return f"--bits {a.bits}: bits per dimension must be in [1, 9]"
    if a.search_mode not in SEARCH_MODES:
        return f"--search_mode {a.search_mode}: one of {', '.join(SEARCH_MODES)}"
    if a.topk < 1 or a.batch < 1 or a.nprobe < 1 or a.nlist < 1 or a.rerank < 0:
        return "--topk, --batch, --nprobe, --nlist must be >= 1 and --rerank >= 0"
    return ""


def log(msg: str) -> None:
    print(f"[rbq] {msg}", file=sys.stderr, flush=True)


def main(argv=None) -> int:
    a = parse_args(argv)
    err = check_args(a)
    if err:
        print(err, file=sys.stderr)
        return 2
    if a.gpus > 1 and "WORLD_SIZE" not in os.environ:
        return subprocess.call(relaunch_cmd(list(sys.argv[1:] if argv is None else argv), a.gpus, _free_port()))
    import torch
    import torch.distributed as dist

    from . import IndexIVFRaBitQ, read_index, write_index
    from .io import EmbeddingShards, NeighborWriter

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    data = (EmbeddingShards.from_manifest(a.encode_dir) if a.encode_dir
            else EmbeddingShards.from_flat(a.emb, a.n, a.d, np.float16))
    N, D = data.n, data.d
    log(f"N={N} D={D} nlist={a.nlist} nprobe={a.nprobe} topk={a.topk} batch={a.batch} "
        f"rerank={a.rerank} gpus={world}")

    def to_dev(x: np.ndarray) -> torch.Tensor:
        # fp16 rows cross PCIe at half the bytes and are widened on the device
        return torch.from_numpy(np.require(x, requirements=["C", "W"])).to(dev, non_blocking=False).float()

    t0 = time.perf_counter()
    if world > 1:
        from .sharded import ShardedIndexIVFRaBitQ
        index = ShardedIndexIVFRaBitQ(D, a.nlist, seed=a.seed, device=local, kmeans_iters=a.kmeans_iters,
                                      max_train_points_per_cluster=a.train_per_cluster, metric=a.metric,
                                      raw_store=a.raw_store, bits_per_dim=a.bits)
        built = False
    elif a.index and os.path.exists(a.index):
        index = read_index(a.index, device=local, metric=a.metric)
        log(f"loaded {a.index} ({index.ntotal} vectors)")
        built = True
    else:
        index = IndexIVFRaBitQ(D, a.nlist, seed=a.seed, device=local, kmeans_iters=a.kmeans_iters,
                               max_train_points_per_cluster=a.train_per_cluster, metric=a.metric,
                               raw_store=a.raw_store, bits_per_dim=a.bits)
        built = False
    if not built:
        m = min(N, a.train_per_cluster * a.nlist)
        pick = (np.arange(m, dtype=np.int64) * N) // m
        train = data.take(pick, widen=False) if m < N else data.rows(0, N, widen=False)
        index.train(to_dev(train))
        for off in range(0, N, a.stream_batch):
            index.add(to_dev(data.rows(off, min(N, off + a.stream_batch), widen=False)))
        torch.cuda.synchronize(dev)
        log(f"built in {time.perf_counter() - t0:.1f} s")
        if a.index and world == 1:
            write_index(index, a.index)
            log(f"saved {a.index}")
    index.nprobe = a.nprobe
    index.k_rerank = a.rerank
    index.prune = a.strategy != "none"
    index.query_bits = SEARCH_MODES[a.search_mode]

    t1 = time.perf_counter()
    writer = NeighborWriter(a.out_nbr, a.out_dist, a.topk) if rank == 0 else None
    for off in range(0, N, a.batch):
        q = to_dev(data.rows(off, min(N, off + a.batch), widen=False))
        dd, ii = index.search(q, a.topk)
        if writer is not None:
            writer.write(ii.cpu().numpy(), dd.cpu().numpy())
        if (off // a.batch) % 50 == 0:
            log(f"searched {min(N, off + a.batch)} / {N}")
    if writer is not None:
        writer.close()
        log(f"search+write {time.perf_counter() - t1:.1f} s -> {a.out_nbr}, {a.out_dist}")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
