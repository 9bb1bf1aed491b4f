"""ctypes binding of the C ABI declared in ``include/ssla_b200.h``.

The library is the only compute path: if ``libssla_b200.so`` is missing or a tensor is not
on a CUDA device the call raises; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "libssla_b200.so"
_lock = threading.Lock()
_lib = None

F32, BF16, F16 = 0, 1, 2
_DT = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}

p, i64, i32, f32, sz = C.c_void_p, C.c_int64, C.c_int, C.c_float, C.c_size_t

# name -> (restype, argtypes); one entry per declaration of include/ssla_b200.h
SIGNATURES = {
    "ssla_abi_version": (i32, []),
    "ssla_last_error": (C.c_char_p, []),
    "ssla_scan_fwd": (i32, [p, i32, p, i32, p, i32, p, i64, i64, i64, p]),
    "ssla_scan_bwd": (i32, [p, i32, p, i32, p, i32, p, i32, p, i32, p, i64, i64, i64, p]),
    "ssla_gla_scalar_fwd": (i32, [p, p, p, p, i32, i32, p, i64, i64, i64, f32, p, p, p, p]),
    "ssla_gla_scalar_bwd": (i32, [p, p, p, p, i32, i32, p, i64, i64, i64, f32, p, p, p, p, p, p, p, p, p]),
    "ssla_recurrent_gla_fwd": (i32, [p, p, p, p, i32, i32, p, i64, i64, i64, i64, i64, f32, p, p, p, p]),
    "ssla_chunk_gla_max_chunks": (i64, [i64, i64]),
    "ssla_chunk_gla_states_bytes": (sz, [i64, i64, i64, i64, i64, i32, i32]),
    "ssla_chunk_gla_workspace_bytes": (sz, [i64, i64, i64, i64, i64, i32, i32]),
    "ssla_chunk_gla_fwd": (
        i32,
        [p, p, p, p, i32, i32, p, i64, i64, i64, i64, i64, f32, p, p, p, p, sz, p, sz, p],
    ),
    "ssla_chunk_gla_bwd": (
        i32,
        [p, p, p, p, i32, i32, p, i64, i64, i64, i64, i64, f32, p, sz, p, p, p, p, p, p, p, p, sz, p],
    ),
    "ssla_chunk_gla_fwd_noalloc": (i32, [p, p, p, p, i32, i32, p, i64, i64, i64, i64, i64, f32, p, p, p, p]),
    "ssla_segment_offsets_sorted": (i32, [p, i64, i64, p, p]),
    "ssla_segment_csr_workspace_bytes": (sz, [i64, i64]),
    "ssla_segment_csr": (i32, [p, i64, i64, p, p, p, sz, p]),
    "ssla_segment_reduce": (i32, [p, i32, p, p, i64, i64, i64, i32, p, p, p]),
    "ssla_gather_rows": (i32, [p, i32, p, i64, i64, p, p]),
    "ssla_scatter_pool_workspace_bytes": (sz, [i64, i64]),
    "ssla_scatter_pool": (i32, [p, i32, p, i64, i64, i64, p, p, p, p, p, p, sz, p]),
    "ssla_index_add_rows_workspace_bytes": (sz, [i64, i64]),
    "ssla_index_add_rows": (i32, [p, i32, p, i64, i64, i64, p, p, sz, p]),
    "ssla_mos_patch_scan_fwd": (i32, [p, p, p, p, i64, i64, p, p]),
    "ssla_mos_patch_scan_routed_fwd": (i32, [p, p, p, i64, i64, p, i64, i64, p, p]),
    "ssla_route_pixel_map": (i32, [p, p, p, i64, i64, i64, i64, p, p, p]),
    "ssla_route_groups_time_sorted": (i32, [p, p, p, i64, p, p]),
    "ssla_route_field_lengths": (i32, [p, p] + [i64] * 11 + [p, p]),
    "ssla_route_compact_fields_workspace_bytes": (sz, [i64]),
    "ssla_route_compact_fields": (i32, [p, i64, p, p, p, p, p, p, sz, p]),
    "ssla_route_fill": (i32, [p, p, p, p] + [i64] * 11 + [p, p, i64, p, p, p, p]),
    "ssla_mos_patch_scan_proj_smem_bytes": (sz, [i64, i64, i64]),
    "ssla_mos_patch_scan_proj_fwd": (i32, [p, i64, p, i64, p, p, p, p, i64, i64, p, p]),
    "ssla_layernorm_residual_fwd": (i32, [p, p, p, p, i64, i64, f32, p, p]),
    "ssla_rows_matmul_smem_bytes": (sz, [i64, i64]),
    "ssla_batched_nms_workspace_bytes": (sz, [i64]),
    "ssla_batched_nms": (i32, [p, p, i64, i64, i32, f32, f32, i64, p, p, p, sz, p]),
    "ssla_dat_window_ranges": (i32, [p, p, p, p, i64, i64, i64, p, p, p]),
    "ssla_dat_decode_windows": (i32, [p, p, p, i64, i64, p, p]),
    "ssla_split_tf32": (i32, [p, i64, p, p, p]),
    "ssla_chunk_gla_tc_timeouts": (i32, [i32, p]),
    "ssla_group_events_workspace_bytes": (sz, [i64, i64, i64, i64]),
    "ssla_group_events_count": (i32, [p, i64, i64, i64, p, i64, i64, i64, i64, p, sz, p, p]),
    "ssla_group_events_emit": (i32, [p, i64, i64, i64, i64, i64, i64, i64, p, i64, i64, i32, p, p, p, p, p, p, p]),
    "ssla_gemm_f32_tc": (i32, [p, i64, i64, i64, p, p, i64, i64, p, i64, p, p]),
    "ssla_rows_matmul_f32": (i32, [p, i64, i64, i64, p, i64, p, i64, p]),
}


def lib_path() -> Path:
    return _LIB_PATH


def load():
    """Load (once) and return the ctypes library handle; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise RuntimeError(
                    f"{_LIB_PATH} is not built; run `python -m ssla_b200.build` "
                    "(ssla_b200 has no CPU fallback)"
                )
            lib = C.CDLL(str(_LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().ssla_last_error().decode(errors="replace")
        if rc == -1:
            raise ValueError(f"{what}: {msg}")
        raise RuntimeError(f"{what} failed ({rc}): {msg}")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}; expected float32, bfloat16 or float16") from None


def ptr(t):
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*ts, what: str = "ssla_b200") -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(f"{what}: tensors must be on a CUDA device (no CPU path)")


def tc_wait_timeouts(reset: bool = True) -> int:
    """Bounded barrier waits of the tensor-core chunk kernels that gave up since the last reset
    (a device read; 0 in a healthy run)."""
    n = C.c_uint(0)
    check(load().ssla_chunk_gla_tc_timeouts(1 if reset else 0, C.addressof(n)), "chunk_gla_tc_timeouts")
    return int(n.value)
