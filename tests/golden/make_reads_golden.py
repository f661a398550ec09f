"""Generate tests/golden/reads_golden.npz: outputs of the reference's own read-to-embedding code
(PoreModel.sequence_to_signal, tile_read, SignalEncoder with a seeded random init,
SignalEvalModel's window preprocessing and AveragePooler), which bench_reads.py restates for
benchmark configuration 3.  Run in a checkout that has the reference's src/ importable:

    python tests/golden/make_reads_golden.py /path/to/reference/src

Everything runs on the CPU in fp32."""
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

src = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_SRC", "")
sys.path.insert(0, src)
from neurosamble.model.pooling import AveragePooler  # noqa: E402
from neurosamble.model.pore_model import PoreModel  # noqa: E402
from neurosamble.model.signal_encoder import SignalEncoder  # noqa: E402
from neurosamble.overlap.eval_model import SignalEvalModel  # noqa: E402
from neurosamble.overlap.tile import tile_read  # noqa: E402

ENC_SEED = 4242
rng = np.random.default_rng(7)
codes = rng.integers(0, 4, 400).astype(np.int8)
seq = "".join("ACGT"[c] for c in codes)
signal = PoreModel(kmer_table_path=None).sequence_to_signal(seq)
lengths = np.array([0, 999, 1000, 1999, 2000, 2999, 3000, 3600, 44955], np.int64)
offsets = [np.array([(o, len(w)) for o, w in tile_read(np.zeros(n, np.float32))], np.int64).reshape(-1, 2)
           for n in lengths]

torch.manual_seed(ENC_SEED)
enc = SignalEncoder(embedding_dim=256, num_heads=8).eval()
model = SignalEvalModel(enc, AveragePooler(), "cpu", embedding_dim=256, use_amp=False)
wrng = np.random.default_rng(11)
wins = [(90 + 20 * wrng.standard_normal(v)).astype(np.float32) for v in (2000, 1500, 1000, 1733)]
emb = model.encode(wins)
sig_b, mask_b = model._prep_batch(wins)

np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "reads_golden.npz"),
                    codes=codes, signal=signal, lengths=lengths,
                    offsets=np.concatenate(offsets), offsets_count=np.array([len(o) for o in offsets]),
                    enc_seed=np.array(ENC_SEED), windows=np.concatenate(wins),
                    window_lengths=np.array([len(w) for w in wins]), prepped=sig_b.numpy(),
                    mask_t=mask_b.numpy(), embeddings=emb,
                    weights_checksum=np.array([float(p.double().sum()) for p in enc.parameters()]))
print("wrote reads_golden.npz", emb.shape)
