from .guard import input_guard, prepare_cu_seqlens

__all__ = ["input_guard", "prepare_cu_seqlens"]
