"""Inputs of benchmark configuration 3 (read-overlap retrieval): simulated nanopore-style reads
of a random genome, turned into current signals and embedded by a seeded, randomly initialised
signal encoder.  This is input generation for bench.py and the tests only; the library
(neurosamble_b200/) never imports it.

The steps restate the reference pipeline that produces the vectors its overlap search indexes:

  genome      seeded uniform A/C/G/T, 10 Mbp
  reads       200,000 x 5,000 bp, uniform start, 50 % reverse-complemented, 8 % errors split
              4 : 2 : 2 between substitution, insertion (a random base after the template base)
              and deletion
  signal      PoreModel.sequence_to_signal (src/neurosamble/model/pore_model.py:93-106): one
              current level per 6-mer, held for 9 samples; without a k-mer table the
              reference uses its synthetic levels (pore_model.py:81-85), restated in kmer_levels
  windows     tile_read (src/neurosamble/overlap/tile.py:22-54): 2,000-sample windows every
              1,000 samples, a trailing partial window kept when it has >= 1,000 samples
  encoder     SignalEvalModel._prep_batch / encode (src/neurosamble/overlap/eval_model.py:90-146):
              z-normalise each window over its valid samples (std floored at 1e-6, padding
              zero), T-resolution mask clamp(valid // 5, 1, 400), SignalEncoder forward
              (src/neurosamble/model/signal_encoder.py:51-180, restated in SignalEncoder below
              with d = 256 and 8 heads), fp16 autocast, AveragePooler (model/pooling.py:17-21),
              L2-normalise
  read vector the mean of the read's window embeddings, L2-normalised, stored as fp16 and read
              back as fp32 (one vector per read; the reference indexes every window)

Everything runs on one CUDA device with torch; reads are processed in fixed batches, so a
read's vector does not depend on how many processes share the work.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

KMER = 6
SAMPLES_PER_KMER = 9
WIN = 2000
STRIDE = 1000
DOWNSAMPLE = 5
BASES = "ACGT"


def kmer_levels(k: int = KMER, mean: float = 90.0, std: float = 20.0) -> np.ndarray:
    """Synthetic pore-model level of every k-mer (index sum_j b_j 4^(k-1-j), A=0 C=1 G=2 T=3):
    mean + (u - 0.5) * 2 * std with u = (first 8 hex digits of md5(kmer) mod 100000) / 100000,
    the reference's fallback when no k-mer table is given."""
    out = np.empty(4 ** k, np.float32)
    for i in range(4 ** k):
        kmer = "".join(BASES[(i >> (2 * (k - 1 - j))) & 3] for j in range(k))
        h = int(hashlib.md5(kmer.encode()).hexdigest()[:8], 16)
        out[i] = np.float32(mean + ((h % 100000) / 100000.0 - 0.5) * 2.0 * std)
    return out


def sequence_to_signal(codes: np.ndarray, levels: np.ndarray) -> np.ndarray:
    """Base codes (0..3) -> piecewise-constant signal: the level of each k-mer held
    SAMPLES_PER_KMER samples."""
    codes = np.asarray(codes, np.int64)
    if codes.size < KMER:
        return np.zeros(0, np.float32)
    idx = np.zeros(codes.size - KMER + 1, np.int64)
    for j in range(KMER):
        idx = idx * 4 + codes[j:codes.size - KMER + 1 + j]
    return np.repeat(levels[idx], SAMPLES_PER_KMER).astype(np.float32)


def window_offsets(n: int, win: int = WIN, stride: int = STRIDE) -> list:
    """(offset, length) of tile_read's windows over a signal of n samples."""
    out, off = [], 0
    while off < n:
        if off + win <= n:
            out.append((off, win))
            off += stride
        else:
            if n - off >= win // 2:
                out.append((off, n - off))
            break
    return out


class SignalEncoder(nn.Module):
    """Conv front end (1 -> 64 channels, kernel 11; 64 -> 512, kernel = stride = 5), GELU,
    Linear 512 -> d, n pre-norm transformer blocks (GELU feed-forward of 4d), final LayerNorm.
    Submodules are created in the reference's order, so one torch seed gives the reference's
    initial weights."""

    def __init__(self, d: int = 256, heads: int = 8, blocks: int = 6, c1: int = 64, c2: int = 512, k1: int = 11,
                 ds: int = DOWNSAMPLE, dropout: float = 0.1):
        super().__init__()
        self.conv1 = nn.Conv1d(1, c1, kernel_size=k1, stride=1, padding=k1 // 2)
        self.conv2 = nn.Conv1d(c1, c2, kernel_size=ds, stride=ds, padding=0)
        self.act = nn.GELU()
        self.proj = nn.Linear(c2, d)
        self.blocks = nn.ModuleList(
            nn.TransformerEncoderLayer(d_model=d, nhead=heads, dim_feedforward=4 * d, dropout=dropout,
                                       activation="gelu", batch_first=True, norm_first=True)
            for _ in range(blocks))
        self.final_norm = nn.LayerNorm(d)

    def forward(self, signal: torch.Tensor, mask_t: torch.Tensor) -> torch.Tensor:
        x = signal.unsqueeze(1).float()
        x = self.act(self.conv1(x))
        x = self.act(self.conv2(x))
        x = self.proj(x.transpose(1, 2))
        if mask_t.shape[1] == x.shape[1]:
            x = x * mask_t.unsqueeze(-1).to(x.dtype)
        for b in self.blocks:
            x = b(x)
        return self.final_norm(x)


def make_encoder(seed: int, device, d: int = 256, heads: int = 8) -> SignalEncoder:
    torch.manual_seed(seed)
    enc = SignalEncoder(d=d, heads=heads)
    return enc.to(device).eval()


def prep_windows(sig: torch.Tensor, valid: torch.Tensor):
    """z-normalise each row of sig [B, WIN] over its first valid[b] samples (padding stays 0)
    and build the T-resolution mask."""
    L = sig.shape[1]
    m = torch.arange(L, device=sig.device)[None, :] < valid[:, None]
    denom = valid.clamp(min=1)[:, None].to(sig.dtype)
    mean = sig.sum(1, keepdim=True) / denom
    diff = (sig - mean) * m
    std = torch.sqrt((diff * diff).sum(1, keepdim=True) / denom).clamp(min=1e-6)
    T = L // DOWNSAMPLE
    vt = (valid // DOWNSAMPLE).clamp(min=1, max=T)
    mask_t = (torch.arange(T, device=sig.device)[None, :] < vt[:, None]).long()
    return diff / std, mask_t


def encode_windows(enc: SignalEncoder, sig: torch.Tensor, valid: torch.Tensor, amp: bool = True) -> torch.Tensor:
    """[B, WIN] raw windows -> [B, d] L2-normalised window embeddings (AveragePooler)."""
    x, mask_t = prep_windows(sig, valid)
    with torch.no_grad():
        with torch.autocast(device_type=x.device.type, dtype=torch.float16, enabled=amp and x.is_cuda):
            h = enc(x, mask_t)
        h = h.float()
        y = (h * mask_t.unsqueeze(-1)).sum(1) / mask_t.sum(-1).unsqueeze(-1)
    return F.normalize(y, dim=-1)


def simulate_reads(genome: torch.Tensor, n: int, length: int, gen: torch.Generator):
    """n reads of `length` template bases: codes [n, maxlen] (-1 past the end), lengths [n],
    starts [n], strands [n] (True = reverse complement).  Per template base: substitution 4 %
    (a uniformly chosen other base), insertion 2 % (the base, then a random base), deletion 2 %."""
    dev = genome.device
    G = genome.shape[0]
    starts = torch.randint(0, G - length + 1, (n,), generator=gen, device=dev)
    rc = torch.rand(n, generator=gen, device=dev) < 0.5
    tmpl = genome[starts[:, None] + torch.arange(length, device=dev)[None, :]].long()
    tmpl = torch.where(rc[:, None], 3 - tmpl.flip(1), tmpl)
    u = torch.rand((n, length), generator=gen, device=dev)
    shift = torch.randint(1, 4, (n, length), generator=gen, device=dev)
    ins_base = torch.randint(0, 4, (n, length), generator=gen, device=dev)
    sub = u < 0.04
    ins = (u >= 0.04) & (u < 0.06)
    dele = (u >= 0.06) & (u < 0.08)
    base = torch.where(sub, (tmpl + shift) % 4, tmpl)
    cnt = torch.ones_like(tmpl)
    cnt = torch.where(dele, torch.zeros_like(cnt), torch.where(ins, torch.full_like(cnt, 2), cnt))
    pos = torch.cumsum(cnt, 1) - cnt
    lens = cnt.sum(1)
    out = torch.full((n, int(lens.max().item()) + 1), -1, dtype=torch.long, device=dev)
    rows = torch.arange(n, device=dev)[:, None].expand_as(tmpl)
    keep = cnt > 0
    out[rows[keep], pos[keep]] = base[keep]
    out[rows[ins], pos[ins] + 1] = ins_base[ins]
    return out[:, :-1], lens, starts, rc


def read_signals(codes: torch.Tensor, lens: torch.Tensor, levels: torch.Tensor):
    """Base codes [n, maxlen] -> signals [n, (maxlen - KMER + 1) * 9] and their lengths."""
    n, ml = codes.shape
    c = codes.clamp(min=0)
    nk = ml - KMER + 1
    idx = torch.zeros((n, nk), dtype=torch.long, device=codes.device)
    for j in range(KMER):
        idx = idx * 4 + c[:, j:j + nk]
    sig = levels[idx].repeat_interleave(SAMPLES_PER_KMER, dim=1)
    slen = (lens - KMER + 1).clamp(min=0) * SAMPLES_PER_KMER
    return sig, slen


def read_windows(sig: torch.Tensor, slen: torch.Tensor):
    """tile_read over every row: window rows [nw, WIN] (zero past the valid part), valid [nw],
    and the read index of each window.  Full windows start at 0, STRIDE, ... while they fit;
    the next offset gives a partial window when at least WIN / 2 samples remain."""
    dev = sig.device
    n = slen.long()
    nf = torch.where(n >= WIN, (n - WIN) // STRIDE + 1, torch.zeros_like(n))
    rest = n - nf * STRIDE
    part = (rest > 0) & (rest >= WIN // 2)
    cnt = nf + part.long()
    rid = torch.repeat_interleave(torch.arange(n.shape[0], device=dev), cnt)
    first = torch.cumsum(cnt, 0) - cnt
    j = torch.arange(rid.shape[0], device=dev) - first[rid]
    offs = j * STRIDE
    val = torch.minimum(n[rid] - offs, torch.full_like(offs, WIN))
    cols = offs[:, None] + torch.arange(WIN, device=dev)[None, :]
    w = sig[rid[:, None], cols.clamp(max=sig.shape[1] - 1)]
    w = torch.where(torch.arange(WIN, device=dev)[None, :] < val[:, None], w, torch.zeros_like(w))
    return w, val, rid


def make_read_embeddings(n_reads=200_000, read_len=5000, genome_len=10_000_000, seed=3003, device="cuda",
                         d=256, read_batch=512, win_batch=2048, rank=0, world=1, log=None):
    """Config 3 database (= query set): [n_reads, d] float32 on `device` (fp16-rounded), plus
    (starts, strands) of every read.  Rank r of `world` encodes read batches b with b % world == r;
    the caller gathers the rows (every read batch has the same composition whatever the
    world size)."""
    dev = torch.device(device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    genome = torch.randint(0, 4, (genome_len,), generator=gen, device=dev, dtype=torch.uint8)
    levels = torch.from_numpy(kmer_levels()).to(dev)
    enc = make_encoder(seed + 1, dev, d=d)
    X = torch.zeros((n_reads, d), dtype=torch.float32, device=dev)
    starts = torch.empty(n_reads, dtype=torch.long, device=dev)
    strands = torch.empty(n_reads, dtype=torch.bool, device=dev)
    for bi, a in enumerate(range(0, n_reads, read_batch)):
        b = min(n_reads, a + read_batch)
        rgen = torch.Generator(device=dev)
        rgen.manual_seed(seed * 1_000_003 + bi)
        codes, lens, st, rc = simulate_reads(genome, b - a, read_len, rgen)
        starts[a:b], strands[a:b] = st, rc
        if bi % world != rank:
            continue
        sig, slen = read_signals(codes, lens, levels)
        w, val, rid = read_windows(sig, slen)
        emb = torch.empty((w.shape[0], d), dtype=torch.float32, device=dev)
        for c in range(0, w.shape[0], win_batch):
            emb[c:c + win_batch] = encode_windows(enc, w[c:c + win_batch], val[c:c + win_batch])
        acc = torch.zeros((b - a, d), dtype=torch.float32, device=dev)
        acc.index_add_(0, rid, emb)
        X[a:b] = F.normalize(acc / torch.bincount(rid, minlength=b - a).clamp(min=1)[:, None].float(), dim=-1)
        if log and bi % 50 == 0:
            log(f"[reads] batch {bi}: {w.shape[0]} windows")
    return X.half().float(), starts, strands
