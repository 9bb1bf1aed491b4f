from .chunk import chunk_gla
from .chunk_scalar import chunk_gla_scalar
from .fused_recurrent import fused_recurrent_gla

__all__ = ["chunk_gla", "chunk_gla_scalar", "fused_recurrent_gla"]
