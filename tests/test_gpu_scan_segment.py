"""GPU parity of the scan and segment kernels: bit-exact against the CPU oracle / CPU PyTorch."""
import pytest
import torch
import torch.nn.functional as F

from conftest import GOLDEN
from oracle import gla as og
from oracle import segment as oseg

pytestmark = pytest.mark.gpu


def test_scan_golden_bit_exact():
    from ssla_b200.ops.common.scan import scan

    d = torch.load(GOLDEN / "scan_interp.pt")
    u = d["u"].cuda().requires_grad_()
    g = d["g"].cuda().requires_grad_()
    h = scan(u, g, d["cu"].cuda())
    h.backward(d["dh"].cuda())
    assert torch.equal(h.cpu(), d["h"])
    assert torch.equal(u.grad.cpu(), d["du"]) and torch.equal(g.grad.cpu(), d["dg"])


@pytest.mark.parametrize("C", [12, 24, 7, 256])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_scan_many_short_sequences(C, dtype):
    from ssla_b200.ops.common.scan import scan

    gen = torch.Generator().manual_seed(C)
    lens = torch.randint(1, 12, (3000,), generator=gen)
    lens[::97] = 0  # empty sequences
    lens[5] = 300   # one long sequence
    cu = torch.cat([torch.zeros(1, dtype=torch.int64), lens.cumsum(0)])
    T = int(cu[-1])
    u = torch.randn(T, C, generator=gen).to(dtype)
    g = torch.sigmoid(torch.randn(T, C, generator=gen)).to(dtype)
    h_r = og.scan_ref_vectorized(u, g, cu)
    do = torch.randn(T, C, generator=gen).to(dtype)
    du_r, dg_r = og.scan_ref_bwd_vectorized(do, g, h_r, cu)
    uc, gc = u.cuda().requires_grad_(), g.cuda().requires_grad_()
    h = scan(uc, gc, cu.cuda())
    h.backward(do.cuda())
    assert torch.equal(h.cpu(), h_r)
    assert torch.equal(uc.grad.cpu(), du_r) and torch.equal(gc.grad.cpu(), dg_r)


def _pool_case(seed=0, R=20000, S=5000, C=64, dtype=torch.float32, sorted_=True):
    gen = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, S, (R,), generator=gen)
    if sorted_:
        idx = idx.sort().values
    src = torch.randn(R, C, generator=gen)
    src[::7] = src[3]  # ties for max
    return src.to(dtype), idx, S


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("sorted_", [True, False])
def test_scatter_ops_bit_exact(dtype, sorted_):
    from ssla_b200 import torch_scatter as ts
    from ssla_b200.ops import segment as seg

    src, idx, S = _pool_case(dtype=dtype, sorted_=sorted_)
    exp_idx = idx[:, None].expand(-1, src.shape[1])
    out, arg = ts.scatter_max(src.cuda(), exp_idx.cuda(), dim=0, dim_size=S)
    o_r, a_r = oseg.scatter_max(src, idx, S)
    assert torch.equal(out.cpu(), o_r) and torch.equal(arg.cpu(), a_r)
    m = ts.scatter_mean(src.cuda(), exp_idx.cuda(), dim=0, dim_size=S)
    assert torch.equal(m.cpu(), oseg.scatter_mean(src, idx, S))
    s = ts.scatter_sum(src.cuda(), idx.cuda(), dim=0, dim_size=S)
    assert torch.equal(s.cpu(), oseg.scatter_sum_fast(src, idx, S))
    if sorted_:
        off = seg.segment_offsets_sorted(idx.cuda(), S)
        o2, a2 = seg.segment_reduce(src.cuda(), off, None, seg.MAX, want_arg=True)
        assert torch.equal(o2.cpu(), o_r) and torch.equal(a2.cpu(), a_r)


def test_scatter_fp32_matches_cpu_torch_index_add_order():
    from ssla_b200 import torch_scatter as ts

    src, idx, S = _pool_case(seed=3, sorted_=False)
    ref = torch.zeros(S, src.shape[1]).index_add_(0, idx, src)
    assert torch.equal(ts.scatter_sum(src.cuda(), idx.cuda(), dim=0, dim_size=S).cpu(), ref)


def test_index_add_and_gather():
    from ssla_b200.ops import segment as seg

    gen = torch.Generator().manual_seed(1)
    P, D, C = 50000, 9000, 24
    idx = torch.randint(0, D, (P,), generator=gen)
    idx[:40] = 17  # one big segment (> 32 rows: the long rank-sort path)
    src = torch.randn(P, C, generator=gen)
    out = seg.index_add_rows(src.cuda(), idx.cuda(), D)
    ref = torch.zeros(D, C).index_add_(0, idx, src)
    assert torch.equal(out.cpu(), ref)
    gi = torch.randint(0, D, (777,), generator=gen)
    assert torch.equal(seg.gather_rows(ref.cuda(), gi.cuda()).cpu(), ref[gi])


def test_segment_edge_cases():
    from ssla_b200.ops import segment as seg

    idx = torch.zeros(0, dtype=torch.int64).cuda()
    off = seg.segment_offsets_sorted(idx, 3)
    assert off.tolist() == [0, 0, 0, 0]
    out, arg = seg.segment_reduce(torch.zeros(0, 4).cuda(), off, None, seg.MAX, want_arg=True)
    assert out.abs().sum() == 0 and (arg == 0).all()
    off, rows = seg.segment_csr(torch.tensor([2, 2, 0]).cuda(), 4)
    assert off.tolist() == [0, 1, 1, 3, 3] and rows[:3].tolist() == [2, 0, 1]


def test_segment_op_gradients_match_torch():
    """Backward of the differentiable gather / index_add / segment reductions against torch
    autograd of the equivalent CPU operations."""
    from ssla_b200 import torch_scatter as ts
    from ssla_b200.ops import segment as seg

    gen = torch.Generator().manual_seed(5)
    R, S, C = 3000, 700, 8
    idx = torch.randint(0, S, (R,), generator=gen)
    src = torch.randn(R, C, generator=gen, dtype=torch.float64).float()
    gout = torch.randn(S, C, generator=gen)
    for name, ours, ref in (
        ("sum", lambda x: ts.scatter_sum(x, idx.cuda(), dim=0, dim_size=S),
         lambda x: torch.zeros(S, C).index_add(0, idx, x)),
        ("mean", lambda x: ts.scatter_mean(x, idx.cuda(), dim=0, dim_size=S),
         lambda x: torch.zeros(S, C).index_add(0, idx, x) / torch.bincount(idx, minlength=S).clamp(min=1)[:, None]),
        ("max", lambda x: ts.scatter_max(x, idx.cuda(), dim=0, dim_size=S)[0],
         lambda x: torch.zeros(S, C).scatter_reduce(0, idx[:, None].expand(R, C), x, "amax", include_self=False)),
        ("index_add", lambda x: seg.index_add_rows_ad(x, idx.cuda(), S),
         lambda x: torch.zeros(S, C).index_add(0, idx, x)),
    ):
        a = src.cuda().requires_grad_()
        b = src.clone().requires_grad_()
        ours(a).backward(gout.cuda())
        ref(b).backward(gout)
        assert torch.allclose(a.grad.cpu(), b.grad, atol=1e-6), name
    gi = torch.randint(0, R, (900,), generator=gen)
    a = src.cuda().requires_grad_()
    b = src.clone().requires_grad_()
    g2 = torch.randn(900, C, generator=gen)
    seg.gather_rows_ad(a, gi.cuda()).backward(g2.cuda())
    b[gi].backward(g2)
    assert torch.allclose(a.grad.cpu(), b.grad, atol=1e-6)


@pytest.mark.parametrize("k", [2, 4])
def test_c4_pooling_full_size_bit_exact(k):
    """BASELINE config 4 exactly as specified (16 batches x 2 polarity planes at 240x304, ~5% active
    pixels half uniform / half in 20 sigma-8 blobs, Poisson(3) events per pixel, int64 flat
    indices, C=64 bf16): scatter_max values and argmax, scatter_mean and the gather back to the
    rows, through the torch_scatter interface (expanded index, as layers/sparse_pooling.py:33
    calls it) and through the explicit CSR + segment-reduce path; bit-exact against the CPU
    oracle.  The cell ids of rows ordered by pixel are not monotonic (pixel rows wrap inside a
    cell row), so the unsorted (CSR) path is the one that applies; the sorted-segment path is
    checked on the rows stably re-ordered by cell."""
    from ssla_b200 import torch_scatter as ts
    from ssla_b200.ops import segment as seg
    from ssla_b200.synthetic import pooling_rows

    feats, idx, cells = pooling_rows(seed=0)
    inv, S = cells[k]
    R, C = feats.shape
    assert R > 300_000 and C == 64 and feats.dtype == torch.bfloat16
    mx_r, arg_r = oseg.scatter_max(feats, inv, S)
    mean_r = oseg.scatter_mean(feats, inv, S)
    back_r = mx_r[inv]
    f, ic = feats.cuda(), inv.cuda()
    mx, arg = ts.scatter_max(f, ic[:, None].expand(R, C), dim=0, dim_size=S)
    assert torch.equal(mx.cpu(), mx_r) and torch.equal(arg.cpu(), arg_r)
    assert torch.equal(ts.scatter_mean(f, ic[:, None].expand(R, C), dim=0, dim_size=S).cpu(), mean_r)
    assert not bool((inv[1:] >= inv[:-1]).all())
    off, rows = seg.segment_csr(ic, S)
    mx2, arg2 = seg.segment_reduce(f, off, rows, seg.MAX, want_arg=True)
    mn2, _ = seg.segment_reduce(f, off, rows, seg.MEAN)
    assert torch.equal(mx2.cpu(), mx_r) and torch.equal(arg2.cpu(), arg_r) and torch.equal(mn2.cpu(), mean_r)
    assert torch.equal(seg.gather_rows(mx2, ic).cpu(), back_r)
    # the one-pass kernel (max + argmax + mean + gather back)
    res = seg.scatter_pool(f, ic, S, want_back=True, want_arg=True)
    assert torch.equal(res["max"].cpu(), mx_r) and torch.equal(res["arg"].cpu(), arg_r)
    assert torch.equal(res["mean"].cpu(), mean_r) and torch.equal(res["back"].cpu(), back_r)
    # sorted-segment path on the rows re-ordered by cell (stable): same values, argmax mapped back
    perm = torch.sort(inv, stable=True)[1]
    ps = perm.cuda()
    off3 = seg.segment_offsets_sorted(ic[ps], S)
    mx3, arg3 = seg.segment_reduce(f[ps].contiguous(), off3, None, seg.MAX, want_arg=True)
    mn3, _ = seg.segment_reduce(f[ps].contiguous(), off3, None, seg.MEAN)
    assert torch.equal(mx3.cpu(), mx_r) and torch.equal(mn3.cpu(), mean_r)
    a3 = arg3.cpu()
    assert torch.equal(torch.where(a3 < R, perm[a3.clamp(max=R - 1)], a3), arg_r)


@pytest.mark.parametrize("dtype,C", [(torch.bfloat16, 64), (torch.float32, 64), (torch.float16, 256),
                                     (torch.bfloat16, 8), (torch.float32, 4), (torch.bfloat16, 24),
                                     (torch.float32, 12), (torch.float32, 96), (torch.bfloat16, 96),
                                     (torch.float32, 20)])
def test_scatter_pool_one_pass_bit_exact(dtype, C):
    """``ssla_scatter_pool`` (max + argmax + mean + gather back in one pass) against the CPU
    oracle for lane-group widths of 1 to 32 lanes of 16 bytes, power-of-two and not (C=24 bf16:
    3 lanes, C=12 fp32: 3, C=96 fp32: 24, C=96 bf16: 12), the general-width sequence (C=20
    fp32), segments longer than the register slots (sorted through the rank-count path), empty
    segments, ties, and rows with out-of-range ids (ignored; their back row is not written)."""
    from ssla_b200.ops import segment as seg

    gen = torch.Generator().manual_seed(C)
    R, S = 30000, 6000
    idx = torch.randint(0, S, (R,), generator=gen)
    idx[:70] = 11                      # a segment far longer than any lane group
    idx[100:110] = -1                  # out of range: ignored
    idx[200:205] = S
    idx[idx == 5] = 6                  # segment 5 empty
    src = torch.randn(R, C, generator=gen)
    src[::9] = src[4]
    src = src.to(dtype)
    keep = (idx >= 0) & (idx < S)
    rows = keep.nonzero().squeeze(1)
    mx_r, arg_r = oseg.scatter_max(src[rows], idx[rows], S)
    arg_r = torch.where(arg_r < rows.numel(), rows[arg_r.clamp(max=rows.numel() - 1)], torch.full_like(arg_r, R))
    mean_r = oseg.scatter_mean(src[rows], idx[rows], S)
    res = seg.scatter_pool(src.cuda(), idx.cuda(), S, want_back=True, want_arg=True, want_offsets=True)
    assert torch.equal(res["max"].cpu(), mx_r)
    assert torch.equal(res["arg"].cpu(), arg_r)
    assert torch.equal(res["mean"].cpu(), mean_r)
    assert torch.equal(res["back"].cpu()[rows], mx_r[idx[rows]])
    cnt = torch.bincount(idx[rows], minlength=S)
    assert res["offsets"].cpu().tolist() == [0] + torch.cumsum(cnt, 0).tolist()
    # subsets of the outputs
    only_mean = seg.scatter_pool(src.cuda(), idx.cuda(), S, want_max=False)
    assert set(only_mean) == {"mean"} and torch.equal(only_mean["mean"].cpu(), mean_r)


def test_scatter_pool_empty_inputs():
    from ssla_b200.ops import segment as seg

    res = seg.scatter_pool(torch.zeros(0, 64, dtype=torch.bfloat16).cuda(), torch.zeros(0, dtype=torch.int64).cuda(),
                           3, want_arg=True, want_offsets=True)
    assert res["max"].abs().sum() == 0 and res["mean"].abs().sum() == 0
    assert (res["arg"] == 0).all() and res["offsets"].tolist() == [0, 0, 0, 0]
    res = seg.scatter_pool(torch.randn(4, 64).cuda(), torch.tensor([0, 0, 1, 1]).cuda(), 0)
    assert res["max"].shape == (0, 64)


@pytest.mark.parametrize("C", [4, 12, 24, 48, 96, 20])
def test_index_add_rows_widths(C):
    """Deterministic index_add (one-pass kernel in sum mode) against CPU ``index_add_`` for the
    MoS layer widths (fp32, C = 12 / 24 / 48 / 96 give 3 / 6 / 12 / 24 lanes of 16 bytes), a
    general width (C=20) and segments of up to ~30 rows."""
    from ssla_b200.ops import segment as seg

    gen = torch.Generator().manual_seed(100 + C)
    P, D = 60000, 7000
    idx = torch.randint(0, D, (P,), generator=gen)
    idx[:30] = 5
    src = torch.randn(P, C, generator=gen)
    ref = torch.zeros(D, C).index_add_(0, idx, src)
    assert torch.equal(seg.index_add_rows(src.cuda(), idx.cuda(), D).cpu(), ref)


def test_segment_csr_many_blocks():
    """CSR offsets when the segment count needs more than 1024 scan blocks (the chunked
    totals scan): offsets and the ascending row order per segment."""
    from ssla_b200.ops import segment as seg

    gen = torch.Generator().manual_seed(9)
    S = 1024 * 1024 + 4097
    R = 3 * S
    idx = torch.randint(0, S, (R,), generator=gen)
    off, rows = seg.segment_csr(idx.cuda(), S)
    cnt = torch.bincount(idx, minlength=S)
    ref_off = torch.cat([torch.zeros(1, dtype=torch.int64), torch.cumsum(cnt, 0)])
    assert torch.equal(off.cpu(), ref_off)
    assert torch.equal(rows.cpu(), torch.sort(idx, stable=True)[1])
