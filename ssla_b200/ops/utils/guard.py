"""Boundary conventions of the reference operators (utils/ela_utils.py:127-158).

``input_guard`` makes tensor arguments contiguous and runs the call with the inputs' CUDA
device current, so kernels are enqueued on that device's current stream.
"""
from __future__ import annotations

import functools

import torch


def input_guard(fn):
    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        args = tuple(a.contiguous() if isinstance(a, torch.Tensor) else a for a in args)
        kwargs = {k: (v.contiguous() if isinstance(v, torch.Tensor) else v) for k, v in kwargs.items()}
        dev = None
        for a in list(args) + list(kwargs.values()):
            if isinstance(a, torch.Tensor):
                dev = a.device
                break
        if dev is not None and dev.type == "cuda":
            with torch.cuda.device(dev):
                return fn(*args, **kwargs)
        return fn(*args, **kwargs)

    return wrapper


def prepare_cu_seqlens(cu_seqlens: torch.Tensor, device: torch.device) -> torch.Tensor:
    """int64, contiguous, on ``device`` (the kernels read it on the GPU)."""
    if cu_seqlens is None:
        raise ValueError("cu_seqlens is required (packed variable-length layout [T, H, D])")
    if cu_seqlens.dim() != 1 or cu_seqlens.numel() < 1:
        raise ValueError(f"cu_seqlens must be 1-D [N+1], got shape {tuple(cu_seqlens.shape)}")
    return cu_seqlens.to(device=device, dtype=torch.int64).contiguous()
