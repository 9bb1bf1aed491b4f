"""Pin the CPU oracle against golden vectors made by the reference's own code
(tests/golden/make_golden.py), and check the oracle's forms against each other."""
import torch

from conftest import GOLDEN, rel_err
from oracle import gla as og
from oracle import segment as oseg


def test_c1_anchor_naive_recurrent():
    d = torch.load(GOLDEN / "c1_naive_recurrent.pt")
    o, ht = og.naive_gla_recurrent(d["q"], d["k"], d["v"], d["g"], d["cu"], output_final_state=True)
    assert torch.equal(o, d["o"]) and torch.equal(ht, d["ht"])
    # published anchor values of the reference run
    assert abs(float(o.sum()) - 75.838135) < 1e-4
    assert abs(float(ht.norm()) - 51.842117) < 1e-4
    op = og.naive_gla_parallel(d["q"], d["k"], d["v"], d["g"], d["cu"])
    assert rel_err(op, d["o_parallel"]) < 1e-6


def test_chunk_ref_matches_reference_chunk_gla_fwd_bwd():
    d = torch.load(GOLDEN / "chunk_gla_interp.pt")
    q, k, v, g, h0 = (d[n].clone().double().requires_grad_() for n in ("q", "k", "v", "g", "h0"))
    o, ht = og.chunk_gla_ref(q, k, v, g, d["cu"], initial_state=h0, output_final_state=True)
    (o * d["do"].double()).sum().add((ht.double() * d["dht"].double()).sum()).backward()
    # reference Triton kernels (interpreted, fp32) vs float64 oracle
    assert rel_err(o, d["o"]) < 1e-5
    assert rel_err(ht, d["ht"]) < 1e-5
    for name, t in (("dq", q), ("dk", k), ("dv", v), ("dg", g), ("dh0", h0)):
        assert rel_err(t.grad, d[name]) < 1e-5, name


def test_chunk_ref_vs_recurrent_varlen():
    torch.manual_seed(0)
    T, H, K, V = 150, 2, 16, 8
    cu = torch.tensor([0, 1, 70, 150])
    q, k = torch.randn(T, H, K), torch.randn(T, H, K) * 0.25
    v = torch.randn(T, H, V)
    g = torch.nn.functional.logsigmoid(torch.randn(T, H, K)) / 4
    h0 = torch.randn(3, H, K, V)
    o1, h1 = og.naive_gla_recurrent(q, k, v, g, cu, initial_state=h0, output_final_state=True)
    o2, h2 = og.chunk_gla_ref(q, k, v, g, cu, initial_state=h0, output_final_state=True)
    assert rel_err(o2, o1) < 1e-5 and rel_err(h2, h1) < 1e-5


def test_scan_oracle_bit_exact_vs_reference_kernel():
    d = torch.load(GOLDEN / "scan_interp.pt")
    h = og.scan_ref(d["u"], d["g"], d["cu"])
    assert torch.equal(h, d["h"])
    assert torch.equal(og.scan_ref_vectorized(d["u"], d["g"], d["cu"]), d["h"])
    du, dg = og.scan_ref_bwd(d["dh"], d["g"], h, d["cu"])
    assert torch.equal(du, d["du"]) and torch.equal(dg, d["dg"])
    du2, dg2 = og.scan_ref_bwd_vectorized(d["dh"], d["g"], h, d["cu"])
    assert torch.equal(du2, d["du"]) and torch.equal(dg2, d["dg"])


def test_scalar_oracle_vs_reference_naive():
    d = torch.load(GOLDEN / "gla_scalar_naive.pt")
    o, ht = og.naive_gla_recurrent_scalar(d["q"], d["k"], d["v"], d["g"], d["cu"], initial_state=d["h0"],
                                          output_final_state=True)
    assert torch.equal(o, d["o"]) and torch.equal(ht, d["ht"])


def test_segment_oracle_semantics():
    src = torch.tensor([[1.0, -2.0], [3.0, -2.0], [0.5, 7.0], [3.0, 1.0]])
    idx = torch.tensor([0, 0, 2, 0])
    out, arg = oseg.scatter_max(src, idx, 4)
    assert out.tolist() == [[3.0, 1.0], [0.0, 0.0], [0.5, 7.0], [0.0, 0.0]]
    assert arg.tolist() == [[1, 3], [4, 4], [2, 2], [4, 4]]  # first max wins; empty -> R
    m = oseg.scatter_mean(src, idx, 4)
    assert torch.allclose(m[0], torch.tensor([7.0 / 3, -1.0]))
    assert m[1].tolist() == [0.0, 0.0]
    s = oseg.scatter_sum(src, idx, 4)
    assert torch.equal(s, oseg.scatter_sum_fast(src, idx, 4))
    ref = torch.zeros(4, 2).index_add_(0, idx, src)
    assert torch.equal(oseg.index_add_rows(src, idx, 4), ref)


def test_recurrent_step_equals_naive_recurrent():
    """The vectorised one-token step equals the token recurrence on one-token sequences with a
    carried state (the streaming use of BASELINE config 3)."""
    gen = torch.Generator().manual_seed(4)
    N, H, K, V = 7, 3, 8, 5
    S = torch.randn(N, H, K, V, generator=gen)
    for _ in range(3):
        q, k, g = (torch.randn(N, H, K, generator=gen) for _ in range(3))
        v = torch.randn(N, H, V, generator=gen)
        g = torch.nn.functional.logsigmoid(g)
        o_r, S_r = og.naive_gla_recurrent(q, k, v, g, torch.arange(N + 1), initial_state=S, output_final_state=True)
        o, S = og.naive_gla_recurrent_step(q, k, v, g, S)
        assert torch.allclose(o, o_r, rtol=1e-6, atol=1e-6) and torch.allclose(S, S_r, rtol=1e-6, atol=1e-6)


def test_segment_oracle_matches_torch_scatter_reduce():
    """The segment oracle against an independent implementation of the same documented
    semantics: PyTorch's own CPU scatter_reduce (amax / mean / sum with include_self=False,
    empty segments left at 0).  torch_scatter itself is not installed anywhere here."""
    from oracle import segment as oseg

    gen = torch.Generator().manual_seed(9)
    R, C, S = 5000, 16, 1300  # some segments empty
    idx = torch.randint(0, S, (R,), generator=gen)
    src = torch.randn(R, C, generator=gen)
    src[::5] = src[2]  # ties
    ex = idx[:, None].expand(R, C)
    mx, arg = oseg.scatter_max(src, idx, S)
    ref = torch.zeros(S, C).scatter_reduce_(0, ex, src, reduce="amax", include_self=False)
    assert torch.equal(mx, ref)
    # argmax: a row of the segment holding the max, the first such row
    nonempty = torch.bincount(idx, minlength=S) > 0
    a = arg[nonempty]
    assert torch.equal(idx[a], torch.arange(S)[nonempty][:, None].expand_as(a))
    assert torch.equal(src.gather(0, a), mx[nonempty])
    assert (arg[~nonempty] == R).all()
    mean_ref = torch.zeros(S, C).scatter_reduce_(0, ex, src, reduce="mean", include_self=False)
    assert torch.allclose(oseg.scatter_mean(src, idx, S), mean_ref, rtol=1e-6, atol=1e-7)
    sum_ref = torch.zeros(S, C).scatter_reduce_(0, ex, src, reduce="sum", include_self=False)
    assert torch.equal(oseg.scatter_sum_fast(src, idx, S), sum_ref)


def test_routing_oracle_matches_reference_preprocessing():
    """oracle.routing.preprocess against the grouped input the reference model produced
    (MosModel.preprocess_inputs on event_batch(2, seed=7), tests/golden/make_golden_model.py)."""
    from oracle import routing as orr
    from ssla_b200.synthetic import event_batch

    gold = torch.load(GOLDEN / "model_mos_s.pt")
    ev, ln = event_batch(gold["batch"], seed=gold["seed"])
    g = orr.preprocess(ev, ln, (240, 304), 50)
    for k, v in gold["grouped"].items():
        assert torch.equal(g[k].to(v.dtype), v), k
