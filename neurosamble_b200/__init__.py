"""B200-native IVF-RaBitQ retrieval for Neurosamble (CUDA C-ABI library + FAISS-style API)."""
from . import torch_ops  # registers torch.ops.rbq.*
from .index import IndexIVFRaBitQ, read_index, read_reference_index, write_index, write_reference_index

__all__ = ["IndexIVFRaBitQ", "read_index", "write_index", "read_reference_index", "write_reference_index"]
