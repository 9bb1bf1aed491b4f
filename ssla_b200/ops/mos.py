"""Fused inference ops of the MoS attention layer on the ssla_b200 C ABI (fp32).

``patch_scan`` runs the per-patch part of ``MosAttention.forward``
(layers/mos_attention.py:97-136): gather of the projected event row, sigmoid gate, the gated
scan (ops/common/scan.py:35-43 order) and ``q * h``, written straight into the rows of the
gather-projection buffer.  ``layernorm_residual`` is ``nn.LayerNorm(x + r)`` for narrow rows.
Both are forward-only; the layers use them when no gradient is needed.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _lib


def patch_scan(y: torch.Tensor, key: torch.Tensor, dst: torch.Tensor, cu_seqlens: torch.Tensor,
               C: int, z: torch.Tensor) -> torch.Tensor:
    """For each patch sequence and event t: [q|v|g] = y[key[t]]; h = sigmoid(g) h + v;
    z[dst[t]] = q * h.  ``y``: [rows, 3C] fp32, ``z``: [*, C] fp32 (written in place)."""
    _lib.require_cuda(y, key, dst, cu_seqlens, z, what="patch_scan")
    if y.dtype != torch.float32 or z.dtype != torch.float32:
        raise TypeError("patch_scan: fp32 tensors expected")
    if y.shape[-1] != 3 * C or z.shape[-1] != C:
        raise ValueError("patch_scan: y must have 3C columns and z C columns")
    y, z = y.contiguous(), z
    if not z.is_contiguous():
        raise ValueError("patch_scan: z must be contiguous")
    key = key.to(torch.int64).contiguous()
    dst = dst.to(torch.int64).contiguous()
    cu = cu_seqlens.to(torch.int64).contiguous()
    _lib.check(_lib.load().ssla_mos_patch_scan_fwd(y.data_ptr(), key.data_ptr(), dst.data_ptr(), cu.data_ptr(),
                                                   cu.numel() - 1, C, z.data_ptr(), _lib.stream_of(y)),
               "patch_scan")
    return z


def patch_scan_routed(y: torch.Tensor, src: torch.Tensor, pos: Optional[torch.Tensor], P: int, Pg: int,
                      cu_seqlens: torch.Tensor, C: int, z: torch.Tensor) -> torch.Tensor:
    """``patch_scan`` with key = src * P + pos (src when P == 1) and dst = src * Pg + pos (the
    patch event's own row when Pg == 0) formed inside the kernel; ``pos`` may be None when P == 1
    and Pg <= 1."""
    _lib.require_cuda(y, src, cu_seqlens, z, what="patch_scan_routed")
    if y.dtype != torch.float32 or z.dtype != torch.float32:
        raise TypeError("patch_scan_routed: fp32 tensors expected")
    if y.shape[-1] != 3 * C or z.shape[-1] != C or not z.is_contiguous():
        raise ValueError("patch_scan_routed: y must have 3C columns, z C contiguous columns")
    y = y.contiguous()
    src = src.to(torch.int64).contiguous()
    pos = None if pos is None else pos.to(torch.int64).contiguous()
    cu = cu_seqlens.to(torch.int64).contiguous()
    _lib.check(_lib.load().ssla_mos_patch_scan_routed_fwd(y.data_ptr(), src.data_ptr(), _lib.ptr(pos), P, Pg,
                                                          cu.data_ptr(), cu.numel() - 1, C, z.data_ptr(),
                                                          _lib.stream_of(y)), "patch_scan_routed")
    return z


PROJ_SMEM_LIMIT = 112 * 1024  # weights of the in-kernel projection must fit this
# The GEMM-fed patch scan is faster (measured on B200: 2.28e3 vs 2.17e3 SSLA-S frames/s) but
# materialises [events, positions * 3C] fp32 rows; above this size the projection moves into
# the scan kernel instead.
Y_BYTES_LIMIT = 8 << 30


def use_patch_scan_proj(E: int, P: int, C: int, I: int) -> bool:
    """True when the projected rows would exceed Y_BYTES_LIMIT and the weights fit in shared
    memory."""
    return (E * P * 3 * C * 4 > Y_BYTES_LIMIT
            and _lib.load().ssla_mos_patch_scan_proj_smem_bytes(P, C, I) <= PROJ_SMEM_LIMIT)


def patch_scan_proj(x: torch.Tensor, w: torch.Tensor, src: torch.Tensor, pos: torch.Tensor, dst: torch.Tensor,
                    cu_seqlens: torch.Tensor, z: torch.Tensor) -> torch.Tensor:
    """``patch_scan`` with the projection in the kernel: [q|v|g] = w[pos[t]] @ x[src[t]];
    ``x``: [E, I], ``w``: [P, 3C, I], ``z``: [*, C] (written in place)."""
    _lib.require_cuda(x, w, src, pos, dst, cu_seqlens, z, what="patch_scan_proj")
    if x.dtype != torch.float32 or w.dtype != torch.float32 or z.dtype != torch.float32:
        raise TypeError("patch_scan_proj: fp32 tensors expected")
    P, C3, I = w.shape
    C = C3 // 3
    if x.shape[-1] != I or z.shape[-1] != C or not z.is_contiguous():
        raise ValueError("patch_scan_proj: shape mismatch")
    x, w = x.contiguous(), w.contiguous()
    src, pos, dst = (t.to(torch.int64).contiguous() for t in (src, pos, dst))
    cu = cu_seqlens.to(torch.int64).contiguous()
    _lib.check(_lib.load().ssla_mos_patch_scan_proj_fwd(
        x.data_ptr(), I, w.data_ptr(), P, src.data_ptr(), pos.data_ptr(), dst.data_ptr(), cu.data_ptr(),
        cu.numel() - 1, C, z.data_ptr(), _lib.stream_of(x)), "patch_scan_proj")
    return z


ROWS_MATMUL_SMEM = 64 * 1024


def matmul_rows(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a [M, K] @ b [K, N] in fp32: the row kernel for skinny shapes (b fits in shared memory),
    torch.matmul otherwise."""
    K, N = b.shape
    if (a.dtype != torch.float32 or b.dtype != torch.float32 or a.dim() != 2 or a.stride(1) != 1
            or _lib.load().ssla_rows_matmul_smem_bytes(K, N) > ROWS_MATMUL_SMEM):
        return a @ b
    _lib.require_cuda(a, b, what="matmul_rows")
    b = b.contiguous()
    out = torch.empty((a.shape[0], N), device=a.device, dtype=torch.float32)
    _lib.check(_lib.load().ssla_rows_matmul_f32(a.data_ptr(), a.shape[0], K, a.stride(0), b.data_ptr(), N,
                                                out.data_ptr(), N, _lib.stream_of(a)), "matmul_rows")
    return out


def layernorm_residual(x: torch.Tensor, r: Optional[torch.Tensor], weight: torch.Tensor, bias: torch.Tensor,
                       eps: float) -> torch.Tensor:
    """LayerNorm(x + r) * weight + bias over the last dimension (fp32, forward only)."""
    _lib.require_cuda(x, weight, bias, what="layernorm_residual")
    C = x.shape[-1]
    x = x.contiguous()
    r = None if r is None else r.contiguous()
    out = torch.empty_like(x)
    _lib.check(_lib.load().ssla_layernorm_residual_fwd(
        x.data_ptr(), 0 if r is None else r.data_ptr(), weight.contiguous().data_ptr(), bias.contiguous().data_ptr(),
        x.numel() // max(C, 1), C, float(eps), out.data_ptr(), _lib.stream_of(x)), "layernorm_residual")
    return out


def split_tf32(w: torch.Tensor):
    """(hi, lo) with hi = w rounded to TF32 and lo = w - hi, both fp32 like ``w`` (contiguous):
    the pre-split right-hand operand of ``matmul_tc``."""
    _lib.require_cuda(w, what="split_tf32")
    w = w.contiguous().float()
    hi, lo = torch.empty_like(w), torch.empty_like(w)
    _lib.check(_lib.load().ssla_split_tf32(w.data_ptr(), w.numel(), hi.data_ptr(), lo.data_ptr(), _lib.stream_of(w)),
               "split_tf32")
    return hi, lo


_ERR = {}


def _dev_index(dev) -> int:
    dev = torch.device(dev)
    return dev.index if dev.index is not None else torch.cuda.current_device()


def _err_flag(dev) -> torch.Tensor:
    i = _dev_index(dev)
    f = _ERR.get(i)
    if f is None:
        f = _ERR[i] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", i))
    return f


def tc_gemm_ok(a: torch.Tensor, k: int) -> bool:
    """Whether ``matmul_tc`` takes ``a`` (fp32 rows, 16-byte aligned, K a multiple of 4)."""
    return (a.dtype == torch.float32 and a.dim() == 2 and a.stride(1) == 1 and a.stride(0) % 4 == 0
            and a.data_ptr() % 16 == 0 and k % 4 == 0 and a.shape[1] == k)


def matmul_tc(a: torch.Tensor, bt_split) -> torch.Tensor:
    """a [M, K] @ B^T in fp32 on the tensor cores (split TF32), B given as ``split_tf32`` of
    B [N, K] (or of B zero-padded to [N, 32] when K < 32: whole-row copies).  The device error flag of the kernel's bounded waits is checked lazily by
    ``check_tc_errors``."""
    bh, bl = bt_split
    _lib.require_cuda(a, bh, bl, what="matmul_tc")
    M, K = a.shape
    N = bh.shape[0]
    if not tc_gemm_ok(a, K) or bh.shape[1] < K or bh.shape != bl.shape:
        raise ValueError("matmul_tc: a must be fp32 [M, K] with 16-byte aligned rows, K % 4 == 0, B [N, >= K]")
    out = torch.empty((M, N), device=a.device, dtype=torch.float32)
    _lib.check(_lib.load().ssla_gemm_f32_tc(a.data_ptr(), M, K, a.stride(0), bh.data_ptr(), bl.data_ptr(), N,
                                            bh.shape[1],
                                            out.data_ptr(), N, _err_flag(a.device).data_ptr(), _lib.stream_of(a)),
               "gemm_f32_tc")
    return out


def check_tc_errors(dev) -> None:
    """Raise if a ``matmul_tc`` launch on ``dev`` reported a pipeline timeout (one host read)."""
    f = _ERR.get(_dev_index(dev))
    if f is not None and int(f.item()):
        f.zero_()
        raise RuntimeError("matmul_tc: a tensor-core GEMM pipeline wait timed out")


TC_MIN_ROWS = 4096  # below this the CUDA-core row kernel's single launch is as fast


class RowsGemm:
    """Right-hand operand B [K, N] of ``a @ B`` prepared for both fp32 paths: the tensor-core
    GEMM (``matmul_tc``, B^T split to TF32 once) for many rows with K a multiple of 4, the
    CUDA-core row kernel (``matmul_rows``) otherwise."""

    def __init__(self, b_kn: torch.Tensor):
        self.b = b_kn.contiguous().float()
        self.K = self.b.shape[0]
        bt = self.b.t().contiguous()
        if self.K < 32:  # pad rows to one 128-byte k block: the B tiles then copy whole rows
            bt = torch.nn.functional.pad(bt, (0, 32 - self.K))
        self.split = split_tf32(bt) if self.K % 4 == 0 else None

    def __call__(self, a: torch.Tensor) -> torch.Tensor:
        if self.split is not None and a.shape[0] >= TC_MIN_ROWS and tc_gemm_ok(a, self.K):
            return matmul_tc(a, self.split)
        return matmul_rows(a, self.b)
