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


def _inputs(seed, T, H, K, V, cu, dtype):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(T, H, K, generator=gen).to(dtype).cuda()
    k = (torch.randn(T, H, K, generator=gen) * K ** -0.5).to(dtype).cuda()
    v = torch.randn(T, H, V, generator=gen).to(dtype).cuda()
    g = (F.logsigmoid(torch.randn(T, H, K, generator=gen)) / 16).to(dtype).cuda()
    h0 = (torch.randn(len(cu) - 1, H, K, V, generator=gen) * 0.1).cuda()
    return q, k, v, g, h0, torch.tensor(cu).cuda()


def _regular(L, q, k, v, g, h0, cu, H, K, V, stream):
    """The regular entry point, with caller-allocated states and workspace."""
    from ssla_b200 import _lib

    T, N = q.shape[0], cu.numel() - 1
    dt = _lib.dtype_code(q)
    o = torch.empty_like(v)
    ht = torch.empty(N, H, K, V, device="cuda")
    sb = L.ssla_chunk_gla_states_bytes(N, T, H, K, V, dt, dt)
    states = torch.empty(sb, device="cuda", dtype=torch.uint8)
    nb = L.ssla_chunk_gla_workspace_bytes(N, T, H, K, V, dt, dt)
    ws = torch.empty(nb, device="cuda", dtype=torch.uint8)
    _lib.check(L.ssla_chunk_gla_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(), dt, dt,
                                    cu.data_ptr(), N, T, H, K, V, K ** -0.5, h0.data_ptr(),
                                    o.data_ptr(), ht.data_ptr(), states.data_ptr(), sb, ws.data_ptr(), nb,
                                    stream), "regular")
    return o, ht


def _noalloc(L, q, k, v, g, h0, cu, H, K, V, stream, o, ht):
    from ssla_b200 import _lib

    T, N = q.shape[0], cu.numel() - 1
    dt = _lib.dtype_code(q)
    _lib.check(L.ssla_chunk_gla_fwd_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), g.data_ptr(),
                                            dt, dt, cu.data_ptr(), N, T, H, K, V, K ** -0.5,
                                            h0.data_ptr(), o.data_ptr(), ht.data_ptr(), stream), "noalloc")


# bf16 with K = V = 64 runs the tensor-core kernels; fp32 and K = V = 32 the CUDA-core ones,
# which use the shared scratch in a different layout.
CASES = [
    (torch.bfloat16, 4, 64, 64, ((0, [0, 2048, 4096, 4200]), (1, [0, 1, 700, 5000]))),
    (torch.float32, 2, 32, 32, ((2, [0, 300, 301, 1000]), (3, [0, 64, 900]))),
]


@pytest.mark.parametrize("dtype,H,K,V,calls", CASES)
def test_noalloc_matches_regular_two_calls(dtype, H, K, V, calls):
    from ssla_b200 import _lib

    L = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for seed, cu in calls:
        args = _inputs(seed, cu[-1], H, K, V, cu, dtype)
        o_ref, ht_ref = _regular(L, *args, H, K, V, stream)
        o = torch.empty_like(args[2])
        ht = torch.empty(len(cu) - 1, H, K, V, device="cuda")
        _noalloc(L, *args, H, K, V, stream, o, ht)
        torch.cuda.synchronize()
        assert rel_err(o, o_ref) < 1e-5 and rel_err(ht, ht_ref) < 1e-5
        # warmed up: a further call allocates nothing (caching allocator and device free bytes)
        before = (torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0])
        _noalloc(L, *args, H, K, V, stream, o, ht)
        torch.cuda.synchronize()
        assert (torch.cuda.memory_allocated(), torch.cuda.mem_get_info()[0]) == before
        assert rel_err(o, o_ref) < 1e-5 and rel_err(ht, ht_ref) < 1e-5


def test_noalloc_rejects_oversized_shapes():
    from ssla_b200 import _lib

    L = _lib.load()
    # 65536 sequences x 4 heads x 64 x 64 states need far more than the built-in scratch
    rc = L.ssla_chunk_gla_fwd_noalloc(None, None, None, None, _lib.BF16, _lib.BF16, None, 65536,
                                      65536, 4, 64, 64, 0.125, None, None, None, None)
    assert rc == -3
    assert b"built-in limit" in L.ssla_last_error()
