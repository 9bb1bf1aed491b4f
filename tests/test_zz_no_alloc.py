"""GPU check of ssla_chunk_gla_fwd_noalloc, the chunk_gla forward for callers that cannot
allocate device memory (for example a runtime that owns every allocation and only hands the
library its input and output buffers).  It must give the same results as the regular
ssla_chunk_gla_fwd, which gets a caller-allocated workspace, on two calls in a row (the second
call reuses the built-in scratch left behind by the first), and reject shapes whose scratch
need exceeds the built-in 64 MiB.

This file is named to be collected last, so that a run stopping at the first failure has
already run every other test."""
import pytest
import torch
import torch.nn.functional as F

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _inputs(seed, T, H, K, V, cu):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(T, H, K, generator=gen).to(torch.bfloat16).cuda()
    k = (torch.randn(T, H, K, generator=gen) * K ** -0.5).to(torch.bfloat16).cuda()
    v = torch.randn(T, H, V, generator=gen).to(torch.bfloat16).cuda()
    g = (F.logsigmoid(torch.randn(T, H, K, generator=gen)) / 16).to(torch.bfloat16).cuda()
    h0 = (torch.randn(len(cu) - 1, H, K, V, generator=gen) * 0.1).cuda()
    return q, k, v, g, h0, torch.tensor(cu).cuda()


def _regular(L, q, k, v, g, h0, cu, H, K, V, stream):
    from ssla_b200 import _lib

    T, N = q.shape[0], cu.numel() - 1
    o = torch.empty_like(v)
    ht = torch.empty(N, H, K, V, device="cuda")
    states = torch.empty(L.ssla_chunk_gla_max_chunks(N, T), H, K, V, device="cuda")
    nb = L.ssla_chunk_gla_workspace_bytes(N, T, H, K, V)
    ws = torch.empty(nb, device="cuda", dtype=torch.uint8)
    _lib.check(L.ssla_chunk_gla_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), _lib.BF16,
                                    _lib.BF16, cu.data_ptr(), N, T, H, K, V, K ** -0.5, h0.data_ptr(),
                                    o.data_ptr(), ht.data_ptr(), states.data_ptr(), ws.data_ptr(), nb,
                                    stream), "regular")
    return o, ht


def _noalloc(L, q, k, v, g, h0, cu, H, K, V, stream):
    from ssla_b200 import _lib

    T, N = q.shape[0], cu.numel() - 1
    o = torch.empty_like(v)
    ht = torch.empty(N, H, K, V, device="cuda")
    _lib.check(L.ssla_chunk_gla_fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(),
                                            _lib.BF16, _lib.BF16, cu.data_ptr(), N, T, H, K, V, K ** -0.5,
                                            h0.data_ptr(), o.data_ptr(), ht.data_ptr(), stream), "noalloc")
    return o, ht


def test_noalloc_matches_regular_two_calls():
    from ssla_b200 import _lib

    L = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    H, K, V = 4, 64, 64
    for seed, cu in ((0, [0, 2048, 4096, 4200]), (1, [0, 1, 700, 5000])):
        args = _inputs(seed, cu[-1], H, K, V, cu)
        o_ref, ht_ref = _regular(L, *args, H, K, V, stream)
        o, ht = _noalloc(L, *args, H, K, V, stream)
        torch.cuda.synchronize()
        assert rel_err(o, o_ref) < 1e-5 and rel_err(ht, ht_ref) < 1e-5


def test_noalloc_rejects_oversized_shapes():
    from ssla_b200 import _lib

    L = _lib.load()
    # 65536 sequences x 4 heads x 64 x 64 states need far more than the built-in scratch
    rc = L.ssla_chunk_gla_fwd_noalloc(None, None, None, None, _lib.BF16, _lib.BF16, None, 65536,
                                      65536, 4, 64, 64, 0.125, None, None, None, None)
    assert rc == -3
    assert b"built-in limit" in L.ssla_last_error()
