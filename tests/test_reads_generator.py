"""Benchmark configuration 3's input generator (bench_reads.py) against outputs of the reference's
own code (tests/golden/reads_golden.npz, written by tests/golden/make_reads_golden.py from the
reference's PoreModel, tile_read, SignalEncoder, SignalEvalModel and AveragePooler): the
synthetic pore-model signal and the window offsets must be identical, the seeded encoder must
start from the same weights, and the fp32 window embeddings must agree to 1e-5."""
import os

import numpy as np
import pytest
import torch

import bench_reads as BR

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reads_golden.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def test_pore_model_signal_is_identical(gold):
    sig = BR.sequence_to_signal(gold["codes"].astype(np.int64), BR.kmer_levels())
    assert sig.dtype == np.float32 and np.array_equal(sig, gold["signal"])


def test_window_offsets_follow_tile_read(gold):
    offs = np.split(gold["offsets"], np.cumsum(gold["offsets_count"])[:-1])
    for n, want in zip(gold["lengths"].tolist(), offs):
        got = np.array(BR.window_offsets(n), np.int64).reshape(-1, 2)
        assert np.array_equal(got, want), n
    # the batched tiling of bench_reads gives the same windows
    lens = torch.tensor([n for n in gold["lengths"].tolist() if n > 0])
    sig = torch.arange(int(lens.max()), dtype=torch.float32)[None, :].repeat(len(lens), 1)
    w, val, rid = BR.read_windows(sig, lens)
    k = 0
    for r, n in enumerate(lens.tolist()):
        for off, v in BR.window_offsets(n):
            assert rid[k].item() == r and val[k].item() == v
            assert torch.equal(w[k, :v], sig[r, off:off + v]) and not w[k, v:].any()
            k += 1
    assert k == w.shape[0]


def test_encoder_weights_windows_and_embeddings(gold):
    enc = BR.make_encoder(int(gold["enc_seed"]), "cpu")
    chk = np.array([float(p.detach().double().sum()) for p in enc.parameters()])
    assert np.array_equal(chk, gold["weights_checksum"])  # same initial weights as the reference
    lens = gold["window_lengths"]
    parts = np.split(gold["windows"], np.cumsum(lens)[:-1])
    sig = torch.zeros((len(parts), BR.WIN))
    for i, p in enumerate(parts):
        sig[i, :len(p)] = torch.from_numpy(p)
    val = torch.from_numpy(lens.astype(np.int64))
    x, mask_t = BR.prep_windows(sig, val)
    assert np.allclose(x.numpy(), gold["prepped"], rtol=0, atol=1e-5)
    assert np.array_equal(mask_t.numpy(), gold["mask_t"])
    emb = BR.encode_windows(enc, sig, val, amp=False).numpy()
    assert np.allclose(emb, gold["embeddings"], rtol=0, atol=1e-5)


def test_simulated_reads_have_the_configured_shape():
    gen = torch.Generator().manual_seed(5)
    genome = torch.randint(0, 4, (200_000,), generator=gen, dtype=torch.uint8)
    codes, lens, starts, rc = BR.simulate_reads(genome, 64, 5000, gen)
    assert codes.shape[0] == 64 and ((lens > 4800) & (lens < 5200)).all()
    assert abs(lens.float().mean().item() - 5000) < 25  # 2 % insertions balance 2 % deletions
    assert 0.3 < rc.float().mean().item() < 0.7
    for r in range(64):  # every base code is valid up to the read's length, -1 after it
        row = codes[r]
        assert (row[:lens[r]] >= 0).all() and (row[:lens[r]] < 4).all() and (row[lens[r]:] == -1).all()
    # forward reads start with the genome (matching the first 20 template bases, errors aside)
    fwd = [r for r in range(64) if not rc[r]]
    agree = np.mean([(codes[r, :20] == genome[starts[r]:starts[r] + 20].long()).float().mean().item() for r in fwd])
    assert agree > 0.7
