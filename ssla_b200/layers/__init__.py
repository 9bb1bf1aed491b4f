from .async_sparse_module import AsyncSparseModule
from .linear_attention import LinearAttention
from .mos_attention import MosAttention
from .sparse_pooling import SparseAdaptiveAvgPool, SparseAdaptiveMaxPool, SparseAvgPool, SparseMaxPool, SparsePool
from .temporal_dropout import TemporalDropout

__all__ = ["AsyncSparseModule", "LinearAttention", "MosAttention", "SparsePool", "SparseMaxPool", "SparseAvgPool",
           "SparseAdaptiveMaxPool", "SparseAdaptiveAvgPool", "TemporalDropout"]
