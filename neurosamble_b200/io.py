"""Embedding inputs and neighbour outputs of the retrieval step, in the reference's formats.

* The encoder's shard manifest (``encode_manifest.json``, written by
  src/neurosamble/overlap/encode.py:227-253): ``D``, ``dtype`` ("float16" or "float32") and
  ``shards[i] = {n_rows, emb_file}``; each shard file is a row-major [n_rows, D] array and the
  global row order is the concatenation of the shards in manifest order
  (read the same way by map_full.py:219-235).
* The ``rabitq_search`` input: one flat fp16 [N, D] row-major file (rabitq_search.cu:105-128).
* Its outputs: ``neighbors.i64`` int64 [N, topk] and ``dists.f32`` float32 [N, topk], flat,
  row-major, appended batch by batch (rabitq_search.cu:164-216), which map_full.py:275-279
  memory-maps back.

Rows are handed out as float32 (fp16 files are widened on the device by the caller, or here
on the host); nothing in this module touches the GPU.
"""
from __future__ import annotations

import json
import os
from typing import List

import numpy as np


class EmbeddingShards:
    """Row access across the shards of an encoder manifest (or one flat file)."""

    def __init__(self, mmaps: List[np.ndarray]):
        if not mmaps:
            raise ValueError("no embedding shards")
        d = {m.shape[1] for m in mmaps}
        if len(d) != 1:
            raise ValueError(f"shards disagree on the dimension: {sorted(d)}")
        self.d = d.pop()
        self.dtype = mmaps[0].dtype
        self.mmaps = mmaps
        self.offsets = np.cumsum([0] + [m.shape[0] for m in mmaps])
        self.n = int(self.offsets[-1])

    @classmethod
    def from_manifest(cls, encode_dir: str) -> "EmbeddingShards":
        with open(os.path.join(encode_dir, "encode_manifest.json")) as f:
            man = json.load(f)
        D = int(man["D"])
        dt = np.float16 if man.get("dtype", "float32") == "float16" else np.float32
        mm = []
        for sh in man["shards"]:
            n = int(sh["n_rows"])
            path = os.path.join(encode_dir, sh["emb_file"])
            want = n * D * np.dtype(dt).itemsize
            have = os.path.getsize(path)
            if have < want:
                raise ValueError(f"{path}: {have} bytes, manifest needs {want}")
            mm.append(np.memmap(path, dtype=dt, mode="r", shape=(n, D)) if n else np.empty((0, D), dt))
        return cls(mm)

    @classmethod
    def from_flat(cls, path: str, n: int, d: int, dtype=np.float16) -> "EmbeddingShards":
        want = int(n) * int(d) * np.dtype(dtype).itemsize
        have = os.path.getsize(path)
        if have < want:
            raise ValueError(f"{path}: {have} bytes, need {want} for [{n}, {d}] {np.dtype(dtype).name}")
        return cls([np.memmap(path, dtype=dtype, mode="r", shape=(int(n), int(d)))])

    def rows(self, a: int, b: int, widen: bool = True) -> np.ndarray:
        """Rows [a, b) in global order, as one C-contiguous array (float32 if widen)."""
        if not 0 <= a <= b <= self.n:
            raise IndexError(f"rows [{a}, {b}) outside [0, {self.n})")
        parts = []
        s = int(np.searchsorted(self.offsets, a, side="right") - 1)
        while a < b:
            lo = a - self.offsets[s]
            hi = min(b, self.offsets[s + 1]) - self.offsets[s]
            parts.append(np.asarray(self.mmaps[s][lo:hi]))
            a += hi - lo
            s += 1
        if not parts:
            out = np.empty((0, self.d), self.dtype)
        else:
            out = np.concatenate(parts) if len(parts) != 1 else np.ascontiguousarray(parts[0])
        return out.astype(np.float32) if widen and out.dtype != np.float32 else out

    def take(self, idx, widen: bool = True) -> np.ndarray:
        """Rows at ascending global indices idx (one fancy-indexed read per shard)."""
        idx = np.asarray(idx, np.int64)
        if idx.size and (idx[0] < 0 or idx[-1] >= self.n or np.any(np.diff(idx) < 0)):
            raise IndexError("take: indices must be ascending and inside the data")
        parts = []
        for s, m in enumerate(self.mmaps):
            lo, hi = np.searchsorted(idx, [self.offsets[s], self.offsets[s + 1]])
            if hi > lo:
                parts.append(np.asarray(m[idx[lo:hi] - self.offsets[s]]))
        out = np.concatenate(parts) if parts else np.empty((0, self.d), self.dtype)
        return out.astype(np.float32) if widen and out.dtype != np.float32 else out


class NeighborWriter:
    """Appends [b, topk] batches to ``neighbors.i64`` / ``dists.f32`` (flat, row-major)."""

    def __init__(self, nbr_path: str, dist_path: str, topk: int):
        self.topk = int(topk)
        self.fn = open(nbr_path, "wb")
        self.fd = open(dist_path, "wb")
        self.rows = 0

    def write(self, ids: np.ndarray, dist: np.ndarray) -> None:
        ids = np.ascontiguousarray(ids, np.int64)
        dist = np.ascontiguousarray(dist, np.float32)
        if ids.shape != dist.shape or ids.ndim != 2 or ids.shape[1] != self.topk:
            raise ValueError("batch must be [b, topk] ids and distances")
        self.fn.write(ids.tobytes())
        self.fd.write(dist.tobytes())
        self.rows += ids.shape[0]

    def close(self) -> None:
        self.fn.close()
        self.fd.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def read_neighbors(nbr_path: str, dist_path: str, n: int, topk: int):
    """The memory maps map_full.py opens over the two output files."""
    return (np.memmap(nbr_path, dtype=np.int64, mode="r", shape=(n, topk)),
            np.memmap(dist_path, dtype=np.float32, mode="r", shape=(n, topk)))
