"""``torch.ops.rbq.*``: PyTorch operators over the C ABI of librbq.so.

The reference exposes its CUDA code to Python as JIT-compiled torch extensions
(src/neurosamble/kernels/ops.py:23-68); this path's operators are registered the same way a
torch user finds them, ``torch.ops.rbq.<name>``, each a thin wrapper of one ``rbq_*`` entry
point of include/rbq.h:

  search(h, q, k, nprobe, rerank, prune, probe_split, seeded, query_bits=4)
                                             -> (dist [n, k] f32, ids [n, k] i64)
  rotate(h, x)                               -> xr [n, Dp]                         (rbq_rotate)
  query_prep(h, qr, bits=4)                  -> (planes [n, bits, Dp/32] i32, delta [n], k1 [n])
  coarse(h, qr, nprobe, margin)              -> (probes [n, nprobe] i32, g [n, nprobe] f32)
  scan(h, qr, planes, delta, k1, probes, g, R, prune, slices, cand_cap, tau0)
                                             -> (cand_ids [n, R] i64, cand_dist [n, R] f32)
  bound_seed(h, qr, planes, delta, k1, probes, g, R, cand_cap) -> tau [n] f32
  rerank(h, q, cand_ids, k)                  -> (dist [n, k] f32, ids [n, k] i64)
  merge_results(dist [p, n, k], ids [p, n, k]) -> (dist [n, k], ids [n, k])

``h`` is the index handle as an int (``IndexIVFRaBitQ.handle.value``).  ``query_bits`` of search
is the search mode: 4 (QUANT4), 8 (QUANT8), 16 (LUT16) or 32 (LUT32); ``bits`` of query_prep is
the query code width, 4 or 8, and scan and bound_seed take it from the planes' shape (the stage
operators cover the two popcount modes).  Inputs are CUDA tensors
on the index's device (made contiguous here); outputs are allocated by PyTorch on that device,
and the work is enqueued on ``torch.cuda.current_stream()`` of it, without synchronising.
Distances are squared L2, ascending; missing results have id -1 and distance +inf.  A failed
call raises RuntimeError with the library's message.  Every operator has a fake
implementation, so output shapes propagate under FakeTensorMode and meta tensors.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch
from torch import Tensor
from torch.library import custom_op

from . import _lib

Pair = Tuple[Tensor, Tensor]


def _p(t: Optional[Tensor]) -> Optional[ctypes.c_void_p]:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _st(t: Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _h(handle: int) -> ctypes.c_void_p:
    if not handle:
        raise RuntimeError("rbq: null index handle")
    return ctypes.c_void_p(handle)


def _cuda(t: Tensor, dtype: torch.dtype, name: str) -> Tensor:
    if not t.is_cuda:
        raise RuntimeError(f"rbq: {name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise RuntimeError(f"rbq: {name} must be {dtype}, got {t.dtype}")
    return t.contiguous()


def _dp(d: int) -> int:
    return (d + 31) // 32 * 32


@custom_op("rbq::search", mutates_args=())
def search(handle: int, q: Tensor, k: int, nprobe: int, rerank: int, prune: bool, probe_split: int,
           seeded: int, query_bits: int = 4) -> Pair:
    q = _cuda(q, torch.float32, "q")
    n = q.shape[0]
    sp = _lib.SearchParams()
    _lib.lib().rbq_search_params_default(ctypes.byref(sp))
    sp.n_probes, sp.k, sp.rerank, sp.prune = nprobe, k, rerank, int(prune)
    sp.probe_split, sp.seeded, sp.query_bits = probe_split, seeded, query_bits
    dist = torch.empty((n, k), dtype=torch.float32, device=q.device)
    ids = torch.empty((n, k), dtype=torch.int64, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("rbq_search", _h(handle), ctypes.byref(sp), _p(q), n, _p(dist), _p(ids), _st(q))
    return dist, ids


@search.register_fake
def _(handle, q, k, nprobe, rerank, prune, probe_split, seeded, query_bits=4):
    n = q.shape[0]
    return q.new_empty((n, k)), q.new_empty((n, k), dtype=torch.int64)


@custom_op("rbq::rotate", mutates_args=())
def rotate(handle: int, x: Tensor) -> Tensor:
    x = _cuda(x, torch.float32, "x")
    out = torch.empty((x.shape[0], _dp(x.shape[1])), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        _lib.call("rbq_rotate", _h(handle), _p(x), x.shape[0], _p(out), _st(x))
    return out


@rotate.register_fake
def _(handle, x):
    return x.new_empty((x.shape[0], _dp(x.shape[1])))


def _bits(bits: int) -> int:
    if bits not in (4, 8):
        raise RuntimeError(f"rbq: query bits must be 4 (QUANT4) or 8 (QUANT8), got {bits}")
    return bits


@custom_op("rbq::query_prep", mutates_args=())
def query_prep(handle: int, qr: Tensor, bits: int = 4) -> Tuple[Tensor, Tensor, Tensor]:
    qr = _cuda(qr, torch.float32, "qr")
    n, dp = qr.shape
    planes = torch.empty((n, _bits(bits), dp // 32), dtype=torch.int32, device=qr.device)
    delta = torch.empty(n, dtype=torch.float32, device=qr.device)
    k1 = torch.empty(n, dtype=torch.float32, device=qr.device)
    with torch.cuda.device(qr.device):
        _lib.call("rbq_query_prep", _h(handle), _p(qr), n, _p(planes), _p(delta), _p(k1), bits, _st(qr))
    return planes, delta, k1


@query_prep.register_fake
def _(handle, qr, bits=4):
    n, dp = qr.shape
    return qr.new_empty((n, _bits(bits), dp // 32), dtype=torch.int32), qr.new_empty(n), qr.new_empty(n)


@custom_op("rbq::coarse", mutates_args=())
def coarse(handle: int, qr: Tensor, nprobe: int, margin: int) -> Pair:
    qr = _cuda(qr, torch.float32, "qr")
    n = qr.shape[0]
    probes = torch.empty((n, nprobe), dtype=torch.int32, device=qr.device)
    g = torch.empty((n, nprobe), dtype=torch.float32, device=qr.device)
    with torch.cuda.device(qr.device):
        _lib.call("rbq_coarse", _h(handle), _p(qr), n, nprobe, margin, _p(probes), _p(g), _st(qr))
    return probes, g


@coarse.register_fake
def _(handle, qr, nprobe, margin):
    n = qr.shape[0]
    return qr.new_empty((n, nprobe), dtype=torch.int32), qr.new_empty((n, nprobe))


def _scan_inputs(qr, planes, delta, k1, probes, g):
    return (_cuda(qr, torch.float32, "qr"), _cuda(planes, torch.int32, "planes"),
            _cuda(delta, torch.float32, "delta"), _cuda(k1, torch.float32, "k1"),
            _cuda(probes, torch.int32, "probes"), _cuda(g, torch.float32, "g"))


@custom_op("rbq::scan", mutates_args=())
def scan(handle: int, qr: Tensor, planes: Tensor, delta: Tensor, k1: Tensor, probes: Tensor, g: Tensor, R: int,
         prune: bool, slices: int, cand_cap: int, tau0: Optional[Tensor]) -> Pair:
    qr, planes, delta, k1, probes, g = _scan_inputs(qr, planes, delta, k1, probes, g)
    n, nprobe = probes.shape
    if tau0 is not None:
        tau0 = _cuda(tau0, torch.float32, "tau0")
    ids = torch.empty((n, R), dtype=torch.int64, device=qr.device)
    dist = torch.empty((n, R), dtype=torch.float32, device=qr.device)
    with torch.cuda.device(qr.device):
        _lib.call("rbq_scan", _h(handle), _p(qr), _p(planes), _p(delta), _p(k1), n, _p(probes), _p(g), nprobe,
                  nprobe, _p(tau0), None, None, R, int(prune), slices, cand_cap, _p(ids), _p(dist), None,
                  _bits(planes.shape[1]), _st(qr))
    return ids, dist


@scan.register_fake
def _(handle, qr, planes, delta, k1, probes, g, R, prune, slices, cand_cap, tau0):
    n = probes.shape[0]
    return qr.new_empty((n, R), dtype=torch.int64), qr.new_empty((n, R))


@custom_op("rbq::bound_seed", mutates_args=())
def bound_seed(handle: int, qr: Tensor, planes: Tensor, delta: Tensor, k1: Tensor, probes: Tensor, g: Tensor,
               R: int, cand_cap: int) -> Tensor:
    qr, planes, delta, k1, probes, g = _scan_inputs(qr, planes, delta, k1, probes, g)
    n, nprobe = probes.shape
    tau = torch.empty(n, dtype=torch.float32, device=qr.device)
    with torch.cuda.device(qr.device):
        _lib.call("rbq_bound_seed", _h(handle), _p(qr), _p(planes), _p(delta), _p(k1), n, _p(probes), _p(g),
                  nprobe, nprobe, R, cand_cap, _p(tau), _bits(planes.shape[1]), _st(qr))
    return tau


@bound_seed.register_fake
def _(handle, qr, planes, delta, k1, probes, g, R, cand_cap):
    return qr.new_empty(probes.shape[0])


@custom_op("rbq::rerank", mutates_args=())
def rerank(handle: int, q: Tensor, cand_ids: Tensor, k: int) -> Pair:
    q = _cuda(q, torch.float32, "q")
    cand_ids = _cuda(cand_ids, torch.int64, "cand_ids")
    n, R = cand_ids.shape
    dist = torch.empty((n, k), dtype=torch.float32, device=q.device)
    ids = torch.empty((n, k), dtype=torch.int64, device=q.device)
    with torch.cuda.device(q.device):
        _lib.call("rbq_rerank", _h(handle), _p(q), n, _p(cand_ids), R, k, _p(dist), _p(ids), _st(q))
    return dist, ids


@rerank.register_fake
def _(handle, q, cand_ids, k):
    n = cand_ids.shape[0]
    return q.new_empty((n, k)), q.new_empty((n, k), dtype=torch.int64)


@custom_op("rbq::merge_results", mutates_args=())
def merge_results(dist: Tensor, ids: Tensor) -> Pair:
    dist = _cuda(dist, torch.float32, "dist")
    ids = _cuda(ids, torch.int64, "ids")
    if dist.dim() != 3 or dist.shape != ids.shape:
        raise RuntimeError("rbq: merge_results takes [parts, n, k] distances and ids of one shape")
    p, n, k = dist.shape
    od = torch.empty((n, k), dtype=torch.float32, device=dist.device)
    oi = torch.empty((n, k), dtype=torch.int64, device=dist.device)
    with torch.cuda.device(dist.device):
        _lib.call("rbq_merge_results", _p(dist), _p(ids), p, n, k, _p(od), _p(oi), _st(dist))
    return od, oi


@merge_results.register_fake
def _(dist, ids):
    _, n, k = dist.shape
    return dist.new_empty((n, k)), ids.new_empty((n, k))
