"""Inputs and outputs of the retrieval step in the reference's formats (CPU), and the
rabitq_search-compatible CLI end to end (GPU)."""
import json
import os

import numpy as np
import pytest

from conftest import mixture


def _manifest(tmp_path, parts, dtype="float16"):
    shards = []
    for r, x in enumerate(parts):
        name = f"emb_shard{r}.bin"
        x.astype(np.float16 if dtype == "float16" else np.float32).tofile(tmp_path / name)
        shards.append({"rank": r, "n_rows": int(x.shape[0]), "emb_file": name, "win_file": "w", "rid_file": "r"})
    man = {"n_shards": len(parts), "total_n_windows": int(sum(p.shape[0] for p in parts)), "D": int(parts[0].shape[1]),
           "win": 2000, "stride": 1000, "dtype": dtype, "shards": shards}
    (tmp_path / "encode_manifest.json").write_text(json.dumps(man))


def test_manifest_rows_span_shards(tmp_path):
    from neurosamble_b200.io import EmbeddingShards
    rng = np.random.default_rng(0)
    parts = [rng.standard_normal((n, 16)).astype(np.float32) for n in (5, 0, 9, 3)]
    _manifest(tmp_path, parts)
    es = EmbeddingShards.from_manifest(str(tmp_path))
    full = np.concatenate(parts).astype(np.float16).astype(np.float32)
    assert es.n == 17 and es.d == 16 and es.dtype == np.float16
    for a, b in [(0, 17), (3, 14), (5, 5), (13, 17), (4, 6)]:
        got = es.rows(a, b)
        assert got.dtype == np.float32 and np.array_equal(got, full[a:b])
    assert es.rows(2, 8, widen=False).dtype == np.float16
    pick = np.array([0, 4, 5, 6, 14, 16])
    assert np.array_equal(es.take(pick), full[pick])
    with pytest.raises(IndexError):
        es.rows(10, 18)
    with pytest.raises(IndexError):
        es.take([3, 2])


def test_manifest_float32_and_short_files(tmp_path):
    from neurosamble_b200.io import EmbeddingShards
    x = np.arange(24, dtype=np.float32).reshape(6, 4)
    _manifest(tmp_path, [x], dtype="float32")
    es = EmbeddingShards.from_manifest(str(tmp_path))
    assert es.dtype == np.float32 and np.array_equal(es.rows(0, 6), x)
    (tmp_path / "emb_shard0.bin").write_bytes(b"\0" * 10)
    with pytest.raises(ValueError, match="manifest needs"):
        EmbeddingShards.from_manifest(str(tmp_path))
    f = tmp_path / "flat.f16"
    x.astype(np.float16).tofile(f)
    assert np.array_equal(EmbeddingShards.from_flat(str(f), 6, 4).rows(0, 6), x)
    with pytest.raises(ValueError, match="need"):
        EmbeddingShards.from_flat(str(f), 7, 4)


def test_neighbor_files_round_trip(tmp_path):
    from neurosamble_b200.io import NeighborWriter, read_neighbors
    rng = np.random.default_rng(1)
    ids = rng.integers(-1, 100, (7, 3))
    d = rng.standard_normal((7, 3)).astype(np.float32)
    with NeighborWriter(str(tmp_path / "n.i64"), str(tmp_path / "d.f32"), 3) as w:
        w.write(ids[:4], d[:4])
        w.write(ids[4:], d[4:])
        with pytest.raises(ValueError):
            w.write(ids[:, :2], d[:, :2])
    assert os.path.getsize(tmp_path / "n.i64") == 7 * 3 * 8 and os.path.getsize(tmp_path / "d.f32") == 7 * 3 * 4
    n, dd = read_neighbors(str(tmp_path / "n.i64"), str(tmp_path / "d.f32"), 7, 3)
    assert np.array_equal(n, ids) and np.array_equal(dd, d)


@pytest.mark.parametrize("argv,msg", [
    ([], "need --emb"),
    (["--emb", "x.f16"], "need --emb"),
    (["--emb", "x.f16", "--n", "10", "--bits", "10"], "must be in [1, 9]"),
    (["--emb", "x.f16", "--n", "10", "--bits", "0"], "must be in [1, 9]"),
    (["--emb", "x.f16", "--n", "10", "--search_mode", "LUT64"], "one of QUANT4, QUANT8, LUT16, LUT32"),
    (["--emb", "x.f16", "--n", "10", "--topk", "0"], "--topk"),
])
def test_cli_rejects_unsupported_flags(argv, msg, capsys):
    from neurosamble_b200 import cli
    assert cli.main(argv) == 2
    assert msg in capsys.readouterr().err


def test_cli_defaults_follow_the_reference():
    from neurosamble_b200 import cli
    a = cli.parse_args(["--emb", "e", "--n", "3"])
    assert (a.d, a.nlist, a.nprobe, a.topk, a.bits, a.batch, a.kmeans_iters) == (384, 21185, 384, 128, 1, 16384, 20)
    assert (a.search_mode, a.strategy, a.out_nbr, a.out_dist, a.rerank) == ("QUANT4", "centroid_reorder",
                                                                             "neighbors.i64", "dists.f32", 0)
    assert cli.check_args(a) == ""
    assert cli.check_args(cli.parse_args(["--emb", "e", "--n", "3", "--bits", "4"])) == ""


@pytest.mark.gpu
@pytest.mark.parametrize("metric,rerank", [("l2", 0), ("ip", 40)])
def test_cli_end_to_end_matches_the_library(tmp_path, metric, rerank):
    """fp16 file in, neighbors.i64 / dists.f32 out; equal to the same build and searches made
    through IndexIVFRaBitQ directly; a second run reuses the saved index and writes the same."""
    import torch
    from neurosamble_b200 import IndexIVFRaBitQ, cli
    from neurosamble_b200.io import read_neighbors
    X, _ = mixture(3000, 64, 24, 0.3, 1, seed=4)
    X16 = X.astype(np.float16)
    X16.tofile(tmp_path / "emb.f16")
    args = ["--emb", str(tmp_path / "emb.f16"), "--n", "3000", "--d", "64", "--nlist", "32", "--nprobe", "8",
            "--topk", "10", "--batch", "700", "--stream_batch", "1100", "--kmeans_iters", "5", "--rerank", str(rerank),
            "--metric", metric, "--index", str(tmp_path / "i.rbq"),
            "--out_nbr", str(tmp_path / "n.i64"), "--out_dist", str(tmp_path / "d.f32")]
    assert cli.main(args) == 0
    n1, d1 = (np.array(a) for a in read_neighbors(str(tmp_path / "n.i64"), str(tmp_path / "d.f32"), 3000, 10))
    idx = IndexIVFRaBitQ(64, 32, seed=7, kmeans_iters=5, metric=metric)
    Xd = torch.from_numpy(X16).cuda().float()
    idx.train(Xd)
    for off in range(0, 3000, 1100):
        idx.add(Xd[off:off + 1100])
    idx.nprobe, idx.k_rerank = 8, rerank
    want_d, want_i = [], []
    for off in range(0, 3000, 700):
        d, i = idx.search(Xd[off:off + 700], 10)
        want_d.append(d.cpu().numpy())
        want_i.append(i.cpu().numpy())
    assert np.array_equal(n1, np.concatenate(want_i))
    assert np.array_equal(d1.view(np.uint32), np.concatenate(want_d).view(np.uint32))
    assert (n1[:, 0] == np.arange(3000)).mean() > 0.9  # all-vs-all: a row finds itself first
    assert cli.main(args) == 0  # reuses i.rbq
    n2, d2 = read_neighbors(str(tmp_path / "n.i64"), str(tmp_path / "d.f32"), 3000, 10)
    assert np.array_equal(np.array(n2), n1) and np.array_equal(np.array(d2).view(np.uint32), d1.view(np.uint32))


def test_cli_gpus_relaunches_through_torchrun():
    from neurosamble_b200 import cli
    a = cli.parse_args(["--emb", "x.f16", "--n", "10", "--gpus", "4"])
    assert a.gpus == 4 and cli.check_args(a) == ""
    cmd = cli.relaunch_cmd(["--emb", "x.f16", "--n", "10", "--gpus", "4"], 4, 29555)
    assert cmd[1:3] == ["-m", "torch.distributed.run"]
    assert "--nproc-per-node=4" in cmd and "--master-addr=127.0.0.1" in cmd and "--master-port=29555" in cmd
    assert cmd[cmd.index("-m", 3):][:2] == ["-m", "neurosamble_b200.cli"] and cmd[-2:] == ["--gpus", "4"]
    assert cli.check_args(cli.parse_args(["--emb", "x", "--n", "1", "--gpus", "0"])) == "--gpus must be >= 1"


def test_cli_accepts_every_search_mode():
    from neurosamble_b200 import cli
    for mode in ("QUANT4", "QUANT8", "LUT16", "LUT32"):
        assert cli.check_args(cli.parse_args(["--emb", "x.f16", "--n", "10", "--search_mode", mode])) == ""
    assert cli.SEARCH_MODES == {"QUANT4": 4, "QUANT8": 8, "LUT16": 16, "LUT32": 32}
