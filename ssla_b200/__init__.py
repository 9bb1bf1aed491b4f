"""ssla_b200: B200-native (sm_100a) kernels for SSLA's spatially-sparse gated-linear-attention
hot path, behind the reference's operator and layer interfaces.

Import paths mirror the reference project (``ops.gla.chunk``, ``ops.common.scan``,
``layers.mos_attention`` ...) under the ``ssla_b200`` package.
"""

__all__ = ["chunk_gla", "fused_recurrent_gla", "chunk_gla_scalar", "scan"]


def __getattr__(name):
    if name == "chunk_gla":
        from .ops.gla.chunk import chunk_gla
        return chunk_gla
    if name == "fused_recurrent_gla":
        from .ops.gla.fused_recurrent import fused_recurrent_gla
        return fused_recurrent_gla
    if name == "chunk_gla_scalar":
        from .ops.gla.chunk_scalar import chunk_gla_scalar
        return chunk_gla_scalar
    if name == "scan":
        from .ops.common.scan import scan
        return scan
    raise AttributeError(name)
