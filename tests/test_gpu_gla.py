"""GPU parity of the GLA kernels (chunk_gla, fused_recurrent_gla, chunk_gla_scalar) against the
CPU oracle.  Tolerances (``assert_close``): RMS relative error (utils/ela_utils.py:63-85 style)
below 1e-5 for fp32 inputs and 2e-2 for bf16 inputs, as the north-star bar states, and every
element within 5x that bound of the largest reference magnitude."""
import pytest
import torch
import torch.nn.functional as F

from conftest import GOLDEN, assert_close, rel_err
from oracle import gla as og

pytestmark = pytest.mark.gpu
FP32_TOL, BF16_TOL = 1e-5, 2e-2


@pytest.fixture(autouse=True)
def no_wait_timeouts():
    """Every test leaves the tensor-core chunk kernels' bounded-wait counter at zero."""
    from ssla_b200 import _lib

    _lib.tc_wait_timeouts(reset=True)
    yield
    assert _lib.tc_wait_timeouts(reset=True) == 0


def make(T, H, K, V, cu, dtype, seed=0, h0=True, gscale=16.0):
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(T, H, K, generator=gen)
    k = torch.randn(T, H, K, generator=gen) * K ** -0.5
    v = torch.randn(T, H, V, generator=gen)
    g = F.logsigmoid(torch.randn(T, H, K, generator=gen)) / gscale
    N = len(cu) - 1
    hz = torch.randn(N, H, K, V, generator=gen) * 0.1 if h0 else None
    do = torch.randn(T, H, V, generator=gen)
    dht = torch.randn(N, H, K, V, generator=gen)
    q, k, v, g, do = (x.to(dtype) for x in (q, k, v, g, do))
    return q, k, v, g, hz, do, dht, torch.tensor(cu)


def ref_fwd_bwd(q, k, v, g, h0, do, dht, cu):
    leaves = [x.detach().double().requires_grad_() for x in (q, k, v, g)]
    h0d = h0.double().requires_grad_() if h0 is not None else None
    o, ht = og.chunk_gla_ref(*leaves, cu, initial_state=h0d, output_final_state=True)
    loss = (o.double() * do.double()).sum() + (ht.double() * dht.double()).sum()
    loss.backward()
    grads = [x.grad for x in leaves] + [h0d.grad if h0d is not None else None]
    return o.detach(), ht.detach(), grads


def run_gpu(fn, q, k, v, g, h0, do, dht, cu):
    dev = "cuda"
    qq, kk, vv, gg = (x.to(dev).requires_grad_() for x in (q, k, v, g))
    h0g = h0.to(dev).requires_grad_() if h0 is not None else None
    o, ht = fn(qq, kk, vv, gg, cu.to(dev), initial_state=h0g, output_final_state=True)
    torch.autograd.backward([o, ht], [do.to(dev), dht.to(dev)])
    grads = [qq.grad, kk.grad, vv.grad, gg.grad, h0g.grad if h0g is not None else None]
    return o.detach().cpu(), ht.detach().cpu(), [x.cpu() if x is not None else None for x in grads]


CASES = [
    (64, 2, 32, 32, [0, 20, 64]),
    (200, 3, 64, 64, [0, 1, 2, 66, 130, 200]),  # length-1 sequences, ragged chunks
    (257, 2, 16, 48, [0, 257]),  # K != V, one long sequence
    (95, 4, 32, 16, [0, 0, 31, 31, 95]),  # empty sequences
    (12, 1, 64, 64, [0, 5, 12]),  # shorter than one chunk
]


@pytest.mark.parametrize("T,H,K,V,cu", CASES)
def test_chunk_gla_fp32(T, H, K, V, cu):
    from ssla_b200.ops.gla.chunk import chunk_gla

    args = make(T, H, K, V, cu, torch.float32, seed=T)
    o_r, ht_r, g_r = ref_fwd_bwd(*args)
    o, ht, g = run_gpu(chunk_gla, *args)
    assert_close(o, o_r, FP32_TOL, "o")
    assert_close(ht, ht_r, FP32_TOL, "ht")
    for name, a, b in zip(("dq", "dk", "dv", "dg", "dh0"), g, g_r):
        assert_close(a, b, FP32_TOL, name)


@pytest.mark.parametrize("T,H,K,V,cu", CASES[:3])
def test_chunk_gla_bf16(T, H, K, V, cu):
    from ssla_b200.ops.gla.chunk import chunk_gla

    args = make(T, H, K, V, cu, torch.bfloat16, seed=T + 1)
    o_r, ht_r, g_r = ref_fwd_bwd(*args)
    o, ht, g = run_gpu(chunk_gla, *args)
    assert o.dtype == torch.bfloat16 and ht.dtype == torch.float32
    assert_close(o, o_r, BF16_TOL, "o")
    assert_close(ht, ht_r, BF16_TOL, "ht")
    for name, a, b in zip(("dq", "dk", "dv", "dg", "dh0"), g, g_r):
        assert_close(a, b, BF16_TOL, name)


def test_chunk_gla_golden_reference_kernels():
    """Against the reference's own chunk_gla (Triton, interpreted) outputs and gradients."""
    from ssla_b200.ops.gla.chunk import chunk_gla

    d = torch.load(GOLDEN / "chunk_gla_interp.pt")
    o, ht, g = run_gpu(chunk_gla, d["q"], d["k"], d["v"], d["g"], d["h0"], d["do"], d["dht"], d["cu"])
    assert_close(o, d["o"], FP32_TOL, "o")
    assert_close(ht, d["ht"], FP32_TOL, "ht")
    for name, a in zip(("dq", "dk", "dv", "dg", "dh0"), g):
        assert_close(a, d[name], FP32_TOL, name)


def test_c1_anchor_both_operators():
    from ssla_b200.ops.gla import chunk_gla, fused_recurrent_gla

    d = torch.load(GOLDEN / "c1_naive_recurrent.pt")
    args = [d[n].cuda() for n in ("q", "k", "v", "g")]
    for fn in (chunk_gla, fused_recurrent_gla):
        o, ht = fn(*args, d["cu"].cuda(), output_final_state=True)
        assert_close(o, d["o"], FP32_TOL, "o")
        assert_close(ht, d["ht"], FP32_TOL, "ht")


def test_chunk_gla_strong_decay_exact_path():
    """Decays large enough that the factorised exponent form would overflow: the kernels must
    switch to exact per-element exponents (no inf/nan).  Reference: the fp32 token recurrence
    (the float64 chunk oracle cannot represent these decays)."""
    from ssla_b200.ops.gla.chunk import chunk_gla

    q, k, v, g, h0, do, dht, cu = make(100, 2, 32, 32, [0, 100], torch.float32, seed=5, gscale=0.08)
    leaves = [x.clone().requires_grad_() for x in (q, k, v, g, h0)]
    o_r, ht_r = og.naive_gla_recurrent(*leaves[:4], cu, initial_state=leaves[4], output_final_state=True)
    torch.autograd.backward([o_r, ht_r], [do, dht])
    o, ht, g_ = run_gpu(chunk_gla, q, k, v, g, h0, do, dht, cu)
    assert torch.isfinite(o).all() and all(torch.isfinite(x).all() for x in g_)
    assert rel_err(o, o_r) < 1e-4 and rel_err(ht, ht_r) < 1e-4
    for a, b in zip(g_, leaves):
        assert rel_err(a, b.grad) < 1e-4


@pytest.mark.parametrize("dtype,tol", [(torch.float32, FP32_TOL), (torch.bfloat16, BF16_TOL)])
@pytest.mark.parametrize("K,V", [(32, 32), (64, 64), (16, 32), (20, 24)])
def test_fused_recurrent_vs_naive(dtype, tol, K, V):
    from ssla_b200.ops.gla import fused_recurrent_gla

    cu = [0, 1, 9, 40, 41]
    q, k, v, g, h0, do, dht, cu = make(41, 3, K, V, cu, dtype, seed=K + V)
    o_r, ht_r = og.naive_gla_recurrent(q.float(), k.float(), v.float(), g.float(), cu, initial_state=h0,
                                       output_final_state=True)
    o, ht = fused_recurrent_gla(q.cuda(), k.cuda(), v.cuda(), g.cuda(), cu.cuda(), initial_state=h0.cuda(),
                                output_final_state=True)
    assert o.dtype == dtype
    assert_close(o, o_r, tol, "o")
    assert_close(ht, ht_r, tol, "ht")


def test_fused_recurrent_streaming_equals_one_call():
    """Carrying the final state between T=1 calls (the streaming use of config 3) equals one
    call over the whole sequence."""
    from ssla_b200.ops.gla import fused_recurrent_gla

    N, H, K, V, T = 512, 4, 32, 32, 6
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(N, T, H, K, generator=gen).cuda()
    k = torch.randn(N, T, H, K, generator=gen).cuda()
    v = torch.randn(N, T, H, V, generator=gen).cuda()
    g = F.logsigmoid(torch.randn(N, T, H, K, generator=gen)).cuda() / 16
    cu_all = torch.arange(N + 1).cuda() * T
    flat = lambda x: x.reshape(N * T, H, -1)
    o_all, h_all = fused_recurrent_gla(flat(q), flat(k), flat(v), flat(g), cu_all, output_final_state=True)
    state = None
    cu1 = torch.arange(N + 1).cuda()
    outs = []
    for t in range(T):
        o, state = fused_recurrent_gla(q[:, t], k[:, t], v[:, t], g[:, t], cu1, initial_state=state,
                                       output_final_state=True)
        outs.append(o)
    o_steps = torch.stack(outs, 1).reshape(N * T, H, V)
    assert rel_err(o_steps, o_all) < 1e-6 and rel_err(state, h_all) < 1e-6


def test_fused_recurrent_backward():
    from ssla_b200.ops.gla import fused_recurrent_gla

    args = make(100, 2, 32, 32, [0, 37, 100], torch.float32, seed=9)
    o_r, ht_r, g_r = ref_fwd_bwd(*args)
    o, ht, g = run_gpu(fused_recurrent_gla, *args)
    assert_close(o, o_r, FP32_TOL, "o")
    for name, a, b in zip(("dq", "dk", "dv", "dg", "dh0"), g, g_r):
        assert_close(a, b, FP32_TOL, name)


def test_chunk_gla_scalar_vs_naive():
    from ssla_b200.ops.gla import chunk_gla_scalar

    d = torch.load(GOLDEN / "gla_scalar_naive.pt")
    leaves = [d[n].clone().requires_grad_() for n in ("q", "k", "v", "g", "h0")]
    o_r, ht_r = og.naive_gla_recurrent_scalar(*leaves[:4], d["cu"], initial_state=leaves[4],
                                              output_final_state=True)
    assert rel_err(o_r, d["o"]) == 0.0
    do = torch.randn_like(o_r)
    dht = torch.randn_like(ht_r)
    torch.autograd.backward([o_r, ht_r], [do, dht])
    gl = [d[n].cuda().requires_grad_() for n in ("q", "k", "v", "g", "h0")]
    o, ht = chunk_gla_scalar(*gl[:4], d["cu"].cuda(), initial_state=gl[4], output_final_state=True)
    torch.autograd.backward([o, ht], [do.cuda(), dht.cuda()])
    assert_close(o, d["o"], FP32_TOL, "o")
    assert_close(ht, d["ht"], FP32_TOL, "ht")
    for name, a, b in zip(("dq", "dk", "dv", "dg", "dh0"), gl, leaves):
        assert_close(a.grad, b.grad, FP32_TOL, name)


def test_c2_full_size_bf16():
    """BASELINE config 2 at full size (B=8, H=4, T=2048, K=V=64, bf16, h0) vs the float64
    chunked oracle: outputs, final state and all gradients within 2e-2."""
    from ssla_b200.ops.gla.chunk import chunk_gla

    B, H, T, K = 8, 4, 2048, 64
    cu = (torch.arange(B + 1) * T).tolist()
    args = make(B * T, H, K, K, cu, torch.bfloat16, seed=0)
    o_r, ht_r, g_r = ref_fwd_bwd(*args)
    o, ht, g = run_gpu(chunk_gla, *args)
    assert_close(o, o_r, BF16_TOL, "o")
    assert_close(ht, ht_r, BF16_TOL, "ht")
    for name, a, b in zip(("dq", "dk", "dv", "dg", "dh0"), g, g_r):
        assert_close(a, b, BF16_TOL, name)


def test_chunk_gla_bf16_mixed_tensor_core_and_exact_chunks():
    """bf16 inputs where some chunks have decay ranges beyond the tensor-core kernels'
    single-reference bound: those chunks are flagged and recomputed by the exact kernels."""
    from ssla_b200.ops.gla.chunk import chunk_gla

    T, H, K = 256, 2, 64
    q, k, v, g, h0, do, dht, cu = make(T, H, K, K, [0, 100, 256], torch.float32, seed=11)
    g[128:192] = g[128:192] * 200.0  # strong decays in one chunk of the second sequence
    q, k, v, g, do = (x.to(torch.bfloat16) for x in (q, k, v, g, do))
    leaves = [x.float().clone().requires_grad_() for x in (q, k, v, g)] + [h0.clone().requires_grad_()]
    o_r, ht_r = og.naive_gla_recurrent(*leaves[:4], cu, initial_state=leaves[4], output_final_state=True)
    torch.autograd.backward([o_r, ht_r], [do.float(), dht])
    o, ht, g_ = run_gpu(chunk_gla, q, k, v, g, h0, do, dht, cu)
    assert_close(o, o_r, BF16_TOL, "o")
    assert_close(ht, ht_r, BF16_TOL, "ht")
    for name, a, b in zip(("dq", "dk", "dv", "dg", "dh0"), g_, leaves):
        assert torch.isfinite(a).all(), name
        assert_close(a, b.grad, BF16_TOL, name)


def test_c3_full_size_streaming_bf16():
    """BASELINE config 3 at full size: 65,536 sequences x H=4, K=V=32, bf16 inputs, fp32 state
    carried through 20 one-token calls of fused_recurrent_gla.  Every step's output and the final
    state are checked on a stratified subset of 512 sequences (every 128th) against the token
    recurrence (``naive_gla_recurrent_step``) fed the same bf16 inputs."""
    from ssla_b200.ops.gla import fused_recurrent_gla

    N, H, K, V, STEPS = 65536, 4, 32, 32, 20
    sub = torch.arange(0, N, 128)
    cu = torch.arange(N + 1).cuda()
    state = None
    ref_state = torch.zeros(sub.numel(), H, K, V)
    gen = torch.Generator(device="cuda").manual_seed(0)
    for t in range(STEPS):
        q = torch.randn(N, H, K, device="cuda", generator=gen).to(torch.bfloat16)
        k = torch.randn(N, H, K, device="cuda", generator=gen).to(torch.bfloat16)
        v = torch.randn(N, H, V, device="cuda", generator=gen).to(torch.bfloat16)
        g = (F.logsigmoid(torch.randn(N, H, K, device="cuda", generator=gen)) / 16).to(torch.bfloat16)
        o, state = fused_recurrent_gla(q, k, v, g, cu, initial_state=state, output_final_state=True)
        o_r, ref_state = og.naive_gla_recurrent_step(q[sub].cpu(), k[sub].cpu(), v[sub].cpu(), g[sub].cpu(),
                                                     ref_state)
        assert o.dtype == torch.bfloat16 and state.dtype == torch.float32
        assert_close(o[sub], o_r, BF16_TOL, f"o step {t}")
    assert_close(state[sub], ref_state, BF16_TOL, "final state")
    assert torch.isfinite(state).all()
