"""FAISS-style IVF-RaBitQ index on one B200 (the drop-in for Neurosamble's search call).

Mirrors the index object that src/neurosamble/overlap/map_full.py drives
(``index.nprobe = P`` at map_full.py:283, ``index.search(x, k) -> (D, I)`` at :195-204,
``faiss.read_index`` / ``write_index`` at :281 and index_ivf.py:140, ``train`` / ``add`` /
``ntotal`` at index_ivf.py:119-133): errors raise RuntimeError, missing results have id -1.

Distances are squared L2 ascending (the reference RaBitQ search returns estimated squared
L2, ivf_rabitq.cu:197-354).  ``metric="ip"`` returns ``1 - d/2`` (the inner product of unit
vectors), descending, for callers written against FAISS METRIC_INNER_PRODUCT.

Inputs may be numpy arrays (host) or torch CUDA tensors on the index's device; outputs
follow the input kind.  PyTorch only provides device memory and the current stream; all
compute runs in librbq.so.
"""
from __future__ import annotations

import ctypes
from typing import Tuple

import numpy as np
import torch

from . import _lib

__all__ = ["IndexIVFRaBitQ", "write_index", "read_index"]


def _stream_ptr(device: int) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


class IndexIVFRaBitQ:
    """IVF-RaBitQ index (1-bit codes, or ExRaBitQ with extra bits) with 4-bit query quantisation
    and optional exact rerank.

    Parameters mirror cuvs::neighbors::ivf_rabitq::index_params (ivf_rabitq.hpp:50-103):
    ``nlist`` (n_lists), ``kmeans_iters`` (kmeans_n_iters), ``max_train_points_per_cluster``,
    ``kmeans`` ("balanced": the reference's hierarchical balanced k-means; "lloyd": plain Lloyd);
    a shard of a sharded index also takes ``shard_rank`` / ``shard_count`` and ``shard_policy``
    ("round_robin": list l on rank l % count; "balanced": lists spread by size^2 at the first add);
    ``raw_store`` ("device": the exact rerank's raw fp32 rows in HBM; "host": in pinned host
    memory read over PCIe, for a raw set larger than the GPU's memory); ``bits_per_dim`` (1: 1-bit
    RaBitQ codes; 2..9: ExRaBitQ, the vectors the 1-bit estimate admits are ranked by the
    distance of their (bits_per_dim)-bit codes).
    Search attributes mirror search_params (ivf_rabitq.hpp:178-228) and FAISS: ``nprobe``,
    ``k_rerank`` (exact fp32 rerank depth R, 0 = estimator order as in the reference),
    ``prune`` (RaBitQ error-bound prune), ``probe_split`` (0 = auto), ``seeded`` (two-phase
    scan slices start from the nearest list's bound seed: -1 = auto, on when the probes are split;
    0 off; 1 on), ``query_bits`` (the search mode: 4 QUANT4, the reference CLI's default;
    8 QUANT8; 16 LUT16 and 32 LUT32, the estimate from fp16 / fp32 tables of the float query),
    ``use_graph`` (replay each batch size's search from a captured CUDA graph; small batches),
    ``scan_kind`` (0 auto; 1 the tile scan; 2 the list scan: fixed per-query thresholds, each probed
    list scored against all its queries by an int8 GEMM on the tensor cores).
    """

    def __init__(self, d: int, nlist: int, seed: int = 7, device: int | None = None, kmeans_iters: int = 20,
                 max_train_points_per_cluster: int = 256, shard_rank: int = 0, shard_count: int = 1,
                 metric: str = "l2", shard_policy: str = "round_robin", kmeans: str = "balanced",
                 raw_store: str = "device", bits_per_dim: int = 1, _handle=None):
        if metric not in ("l2", "ip"):
            raise ValueError("metric must be 'l2' or 'ip'")
        self.d = int(d)
        self.nlist = int(nlist)
        self.metric = metric
        self.device = torch.cuda.current_device() if device is None else int(device)
        self.nprobe = 20
        self.k_rerank = 0
        self.prune = True
        self.probe_split = 0
        self.cand_cap = 0
        self.coarse_margin = 0
        self.seeded = -1
        self.query_bits = 4
        self.use_graph = False
        self.scan_kind = 0
        self._h = ctypes.c_void_p()
        if _handle is not None:
            self._h = _handle
            return
        p = _lib.IndexParams()
        _lib.lib().rbq_index_params_default(ctypes.byref(p))
        p.dim, p.n_lists, p.seed = self.d, self.nlist, int(seed)
        p.kmeans_n_iters, p.max_train_points_per_cluster = int(kmeans_iters), int(max_train_points_per_cluster)
        p.device, p.shard_rank, p.shard_count = self.device, int(shard_rank), int(shard_count)
        if shard_policy not in _lib.SHARD_POLICIES:
            raise ValueError(f"shard_policy must be one of {sorted(_lib.SHARD_POLICIES)}")
        p.shard_policy = _lib.SHARD_POLICIES[shard_policy]
        if kmeans not in _lib.KMEANS_KINDS:
            raise ValueError(f"kmeans must be one of {sorted(_lib.KMEANS_KINDS)}")
        p.kmeans_kind = _lib.KMEANS_KINDS[kmeans]
        if raw_store not in _lib.RAW_STORES:
            raise ValueError(f"raw_store must be one of {sorted(_lib.RAW_STORES)}")
        p.raw_store = _lib.RAW_STORES[raw_store]
        p.bits_per_dim = int(bits_per_dim)
        _lib.call("rbq_index_create", ctypes.byref(p), ctypes.byref(self._h))

    # -- lifecycle -----------------------------------------------------------------------
    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                _lib.lib().rbq_index_free(h)
            except Exception:
                pass
            self._h = ctypes.c_void_p()

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def info(self) -> _lib.IndexInfo:
        out = _lib.IndexInfo()
        _lib.call("rbq_index_info", self._h, ctypes.byref(out))
        return out

    @property
    def ntotal(self) -> int:
        return int(self.info().n_total)

    @property
    def is_trained(self) -> bool:
        return bool(self.info().trained)

    # -- data movement -------------------------------------------------------------------
    def _to_device(self, x) -> Tuple[torch.Tensor, bool]:
        """(float32 contiguous CUDA tensor [n, d], input_was_torch_cuda)."""
        if isinstance(x, torch.Tensor):
            on_dev = x.is_cuda
            t = x.to(device=f"cuda:{self.device}", dtype=torch.float32).contiguous()
        else:
            on_dev = False
            a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
            t = torch.from_numpy(a)
            if t.numel() > (1 << 16):
                t = t.pin_memory()
            t = t.to(device=f"cuda:{self.device}", non_blocking=True)
        if t.dim() != 2 or t.shape[1] != self.d:
            raise RuntimeError(f"expected a [n, {self.d}] matrix, got {tuple(t.shape)}")
        return t, on_dev

    # -- build ---------------------------------------------------------------------------
    def train(self, x) -> None:
        """k-means (nlist centroids; balanced unless kmeans="lloyd") on an evenly strided sample
        of at most max_train_points_per_cluster * nlist rows of x."""
        t, _ = self._to_device(x)
        with torch.cuda.device(self.device):
            _lib.call("rbq_train", self._h, _ptr(t), t.shape[0], _stream_ptr(self.device))

    def set_centroids(self, centroids) -> None:
        c = np.ascontiguousarray(np.asarray(
            centroids.detach().cpu() if isinstance(centroids, torch.Tensor) else centroids, dtype=np.float32))
        if c.shape != (self.nlist, self.d):
            raise RuntimeError(f"centroids must be [{self.nlist}, {self.d}]")
        _lib.call("rbq_set_centroids", self._h, c.ctypes.data_as(ctypes.c_void_p), self.nlist)

    def _labels(self, labels, n: int):
        if labels is None:
            return None
        lab = torch.as_tensor(np.asarray(labels.cpu() if isinstance(labels, torch.Tensor) else labels,
                                         dtype=np.int64).astype(np.uint32).view(np.int32))
        lab = lab.to(f"cuda:{self.device}")
        if lab.numel() != n:
            raise RuntimeError("labels must have one entry per row")
        return lab

    def add(self, x, labels=None) -> None:
        """Append rows (ids continue from ntotal); labels (optional) fix their lists."""
        t, _ = self._to_device(x)
        lab = self._labels(labels, t.shape[0])
        with torch.cuda.device(self.device):
            _lib.call("rbq_add", self._h, _ptr(t), t.shape[0], _ptr(lab) if lab is not None else None,
                      _stream_ptr(self.device))

    def build(self, x, centroids=None, labels=None) -> None:
        """train (or the given centroids) + add in one call (rbq_build; ivf_rabitq::build)."""
        t, _ = self._to_device(x)
        c = None
        if centroids is not None:
            c = np.ascontiguousarray(np.asarray(
                centroids.detach().cpu() if isinstance(centroids, torch.Tensor) else centroids, dtype=np.float32))
            if c.shape != (self.nlist, self.d):
                raise RuntimeError(f"centroids must be [{self.nlist}, {self.d}]")
        lab = self._labels(labels, t.shape[0])
        with torch.cuda.device(self.device):
            _lib.call("rbq_build", self._h, _ptr(t), t.shape[0], self.d,
                      c.ctypes.data_as(ctypes.c_void_p) if c is not None else None,
                      _ptr(lab) if lab is not None else None, _stream_ptr(self.device))

    # -- search --------------------------------------------------------------------------
    def search_params(self, k: int) -> _lib.SearchParams:
        sp = _lib.SearchParams()
        _lib.lib().rbq_search_params_default(ctypes.byref(sp))
        sp.n_probes, sp.k, sp.rerank = int(self.nprobe), int(k), int(self.k_rerank)
        sp.prune, sp.probe_split = int(bool(self.prune)), int(self.probe_split)
        sp.cand_cap, sp.coarse_margin = int(self.cand_cap), int(self.coarse_margin)
        sp.seeded = int(self.seeded)
        sp.query_bits = int(self.query_bits)
        sp.graph = int(bool(self.use_graph))
        sp.scan_kind = int(self.scan_kind)
        return sp

    def search(self, x, k: int):
        """Return (D [n, k] float32, I [n, k] int64), FAISS order (distances first)."""
        t, on_dev = self._to_device(x)
        n = t.shape[0]
        sp = self.search_params(k)
        dist = torch.empty((n, k), dtype=torch.float32, device=t.device)
        ids = torch.empty((n, k), dtype=torch.int64, device=t.device)
        with torch.cuda.device(self.device):
            _lib.call("rbq_search", self._h, ctypes.byref(sp), _ptr(t), n, _ptr(dist), _ptr(ids),
                      _stream_ptr(self.device))
        if self.metric == "ip":
            dist = 1.0 - 0.5 * dist
        if on_dev:
            return dist, ids
        return dist.cpu().numpy(), ids.cpu().numpy()

    def search_host(self, x: np.ndarray, k: int):
        """Host-buffer search through the C ABI (rbq_search_host): copies inside the call."""
        a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
        if a.ndim != 2 or a.shape[1] != self.d:
            raise RuntimeError(f"expected a [n, {self.d}] matrix")
        n = a.shape[0]
        sp = self.search_params(k)
        dist = np.empty((n, k), np.float32)
        ids = np.empty((n, k), np.int64)
        with torch.cuda.device(self.device):
            _lib.call("rbq_search_host", self._h, ctypes.byref(sp), a.ctypes.data_as(ctypes.c_void_p), n,
                      dist.ctypes.data_as(ctypes.c_void_p), ids.ctypes.data_as(ctypes.c_void_p),
                      _stream_ptr(self.device))
        if self.metric == "ip":
            dist = 1.0 - 0.5 * dist
        return dist, ids

    # -- introspection -------------------------------------------------------------------
    def rotation(self) -> np.ndarray:
        dp = self.info().padded_dim
        P = np.empty((dp, dp), np.float32)
        _lib.call("rbq_get_rotation", self._h, P.ctypes.data_as(ctypes.c_void_p))
        return P

    def centroids(self):
        inf = self.info()
        C = np.empty((self.nlist, self.d), np.float32)
        Cr = np.empty((self.nlist, inf.padded_dim), np.float32)
        _lib.call("rbq_get_centroids", self._h, C.ctypes.data_as(ctypes.c_void_p), Cr.ctypes.data_as(ctypes.c_void_p))
        return C, Cr

    def export_lists(self):
        inf = self.info()
        n, w = int(inf.n_local), inf.padded_dim // 32
        off = np.empty(self.nlist + 1, np.int64)
        ids = np.empty(n, np.uint32)
        codes = np.empty((n, w), np.uint32)
        fa, fr, fe = (np.empty(n, np.float32) for _ in range(3))
        _lib.call("rbq_export_lists", self._h, *(a.ctypes.data_as(ctypes.c_void_p) for a in (off, ids, codes, fa, fr, fe)))
        out = {"list_off": off, "ids": ids, "codes": codes, "fadd": fa, "frescale": fr, "ferr": fe}
        ex = int(inf.bits_per_dim) - 1
        if ex > 0:
            xc = np.empty((n, ex, w), np.uint32)
            xa, xr = np.empty(n, np.float32), np.empty(n, np.float32)
            _lib.call("rbq_export_ex_lists", self._h, *(a.ctypes.data_as(ctypes.c_void_p) for a in (xc, xa, xr)))
            out.update(ex_bits=ex, ex_codes=xc, fexadd=xa, fexr=xr, ex_scale=float(inf.ex_scale))
        return out

    def list_offsets(self) -> np.ndarray:
        """[nlist + 1] int64: list l holds this shard's slots [off[l], off[l + 1])."""
        off = np.empty(self.nlist + 1, np.int64)
        _lib.call("rbq_export_lists", self._h, off.ctypes.data_as(ctypes.c_void_p), None, None, None, None, None)
        return off

    def list_owners(self) -> np.ndarray:
        """[nlist] int32: the shard holding each list (-1 before a balanced map is fixed)."""
        own = np.empty(self.nlist, np.int32)
        _lib.call("rbq_get_list_owners", self._h, own.ctypes.data_as(ctypes.c_void_p))
        return own

    @property
    def bits_per_dim(self) -> int:
        return int(self.info().bits_per_dim)

    @property
    def query_scale(self) -> float:
        return float(self.info().query_scale)


def write_index(index: IndexIVFRaBitQ, path: str) -> None:
    _lib.call("rbq_save", index.handle, str(path).encode())


def read_index(path: str, device: int | None = None, shard_rank: int = -1, shard_count: int = 0,
               metric: str = "l2") -> IndexIVFRaBitQ:
    dev = torch.cuda.current_device() if device is None else int(device)
    h = ctypes.c_void_p()
    _lib.call("rbq_load", str(path).encode(), dev, int(shard_rank), int(shard_count), ctypes.byref(h))
    out = _lib.IndexInfo()
    _lib.call("rbq_index_info", h, ctypes.byref(out))
    return IndexIVFRaBitQ(out.dim, out.n_lists, device=dev, metric=metric, _handle=h)


def read_reference_index(path: str, X=None, device: int | None = None, shard_rank: int = 0, shard_count: int = 1,
                         shard_policy: str = "round_robin", metric: str = "l2") -> IndexIVFRaBitQ:
    """Import an index file written by the reference (cuVS ivf_rabitq serialize / IVFGPU::save,
    1-bit codes, matmul rotator).  X (optional, [num_vectors, D] float32, row = id) supplies
    the raw vectors of the exact rerank; without it the index searches with k_rerank = 0."""
    dev = torch.cuda.current_device() if device is None else int(device)
    xh = None
    n_x = 0
    if X is not None:
        xh = np.ascontiguousarray(X.cpu().numpy() if isinstance(X, torch.Tensor) else X, dtype=np.float32)
        n_x = xh.shape[0]
    h = ctypes.c_void_p()
    _lib.call("rbq_import_reference", str(path).encode(), dev,
              xh.ctypes.data_as(ctypes.c_void_p) if xh is not None else None, n_x, int(shard_rank),
              int(shard_count), _lib.SHARD_POLICIES[shard_policy], ctypes.byref(h))
    out = _lib.IndexInfo()
    _lib.call("rbq_index_info", h, ctypes.byref(out))
    return IndexIVFRaBitQ(out.dim, out.n_lists, device=dev, metric=metric, _handle=h)


def write_reference_index(index: IndexIVFRaBitQ, path: str) -> None:
    """Write an unsharded index in the reference's file format (IVFGPU::save)."""
    _lib.call("rbq_export_reference", index.handle, str(path).encode())
