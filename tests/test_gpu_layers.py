"""GPU parity of the routing, layers and the full SSLA model against fixtures produced by the
reference's own Python implementation (tests/golden/make_golden_model.py).  Integer routing
outputs must match exactly; floating-point layer outputs within 1e-5 relative (fp32)."""
import pytest
import torch
import yaml

from conftest import GOLDEN, ROOT, assert_close, rel_err

pytestmark = pytest.mark.gpu
FP32_TOL = 1e-5

CFG = {
    "S": {"name": "MOS_S", "expected_strides": [8], "layers": [
        {"name": "MosAttention", "kernel_size": 1, "hidden_size": 12},
        {"name": "MosAttention", "kernel_size": 3, "hidden_size": 12},
        {"name": "SparseMaxPool", "kernel_size": 2}, {"name": "TemporalDropout", "window_size": 4},
        {"name": "MosAttention", "kernel_size": 3, "hidden_size": 24},
        {"name": "MosAttention", "kernel_size": 3, "hidden_size": 24},
        {"name": "SparseMaxPool", "kernel_size": 2}, {"name": "TemporalDropout", "window_size": 4},
        {"name": "MosAttention", "kernel_size": 3, "hidden_size": 48},
        {"name": "MosAttention", "kernel_size": 3, "hidden_size": 48},
        {"name": "SparseMaxPool", "kernel_size": 2}, {"name": "TemporalDropout", "window_size": 4},
        {"name": "MosAttention", "kernel_size": 3, "hidden_size": 96},
        {"name": "MosAttention", "kernel_size": 3, "hidden_size": 96}]},
}
CFG["L"] = {"name": "MOS_L", "expected_strides": [8], "layers": [
    dict(l, hidden_size={12: 32, 24: 64, 48: 128, 96: 256}[l["hidden_size"]]) if "hidden_size" in l else l
    for l in CFG["S"]["layers"]]}


def _model(variant):
    from ssla_b200.model import MosDetector
    from ssla_b200.synthetic import seeded_parameters

    m = MosDetector(CFG[variant], dataset="Gen1", hot_pixel_thres=50)
    seeded_parameters(m, 2025)
    return m.cuda().eval()


def _events(B):
    from ssla_b200.synthetic import event_batch

    ev, ln = event_batch(B, seed=7)
    return ev.cuda(), ln.cuda()


@pytest.fixture(scope="module")
def gold_s():
    return torch.load(GOLDEN / "model_mos_s.pt")


def test_preprocess_exact(gold_s):
    from ssla_b200.model import preprocess_inputs

    ev, ln = _events(gold_s["batch"])
    x = preprocess_inputs(ev, ln, (240, 304), 50)
    for k, v in gold_s["grouped"].items():
        assert torch.equal(x[k].cpu().to(v.dtype), v), k


def test_patch_routing_exact(gold_s):
    from ssla_b200.utils.async_utils import get_patch2pixel_lut, scatter_group_events_to_patch

    g = {k: v.cuda().to(torch.int64) if k != "events" else v.cuda() for k, v in gold_s["grouped"].items()}
    g["batch_size"] = gold_s["batch"]
    lut = get_patch2pixel_lut((240, 304), (3, 3), (1, 1)).cuda()
    p = scatter_group_events_to_patch(g, (240, 304), lut)
    ref = gold_s["patch"]
    assert torch.equal(p["lengths"].cpu().to(torch.int32), ref["lengths"])
    assert torch.equal(p["orig_event_idx"].cpu().to(torch.int32), ref["orig_event_idx"])
    assert torch.equal(p["pos_id"].cpu().to(torch.int8), ref["pos_id"])
    assert torch.equal(p["events"].cpu(), g["events"].cpu()[p["orig_event_idx"].cpu()])


def test_receptive_field_routing_exact(gold_s):
    from ssla_b200.utils.farsecnn_utils import compute_rf2pixels, gather_receptive_fields

    g = {k: v.cuda().to(torch.int64) for k, v in gold_s["grouped"].items() if k != "events"}
    g["events"] = gold_s["layer1"]["events"].cuda()
    g["batch_size"] = gold_s["batch"]
    lut, oc = compute_rf2pixels((240, 304), (2, 2), (2, 2))
    rf = gather_receptive_fields(g, (240, 304), lut.cuda(), oc.cuda(), kernel_size=(2, 2), stride=(2, 2))
    for k, v in gold_s["rf2x2"].items():
        got = rf[k].cpu()
        assert torch.equal(got.to(v.dtype), v), k


@pytest.mark.parametrize("variant", ["S", "L"])
def test_full_model_matches_reference(variant, gold_s):
    """Preprocessing, every MoS attention / sparse max-pool / temporal-dropout layer, grid
    densification and the YOLOX head decode, against the reference model on the CPU."""
    gold = gold_s if variant == "S" else torch.load(GOLDEN / "model_mos_l.pt")
    m = _model(variant)
    ev, ln = _events(gold["batch"])
    from ssla_b200.model import async_event_to_grid, preprocess_inputs

    with torch.no_grad():
        x = preprocess_inputs(ev, ln, m.frame_size, m.hot_pixel_thres)
        taps = []
        for i, layer in enumerate(m.backbone):
            x = layer(x)
            if f"layer{i}" in gold:
                ref = gold[f"layer{i}"]
                assert torch.equal(x["lengths"].cpu().to(torch.int32), ref["lengths"]), i
                assert torch.equal(x["time"].cpu().to(torch.int32), ref["time"]), i
                assert rel_err(x["events"], ref["events"]) < FP32_TOL, i
            if i in m.output_indices:
                taps.append(x)
        grids = [async_event_to_grid(t, m.grid_sizes[k], m.in_features[k]) for k, t in enumerate(taps)]
        for a, b in zip(grids, gold["grids"]):
            assert rel_err(a, b) < FP32_TOL
        torch.backends.cudnn.allow_tf32 = False
        head = m.head(grids)
    # the head decode exponentiates box sizes (x up to ~300): 1e-4 relative for the dense head
    assert head.shape == gold["head"].shape
    assert rel_err(head, gold["head"]) < 1e-4


def test_full_model_s_batch8_matches_reference():
    """SSLA-S at batch 8 (the per-GPU share of BASELINE config 5's batch of 64 on 8 GPUs): backbone
    grids and head output against the reference MosModel on the CPU
    (tests/golden/make_golden_model.py --batch8: event_batch(8, seed=21), weights seed 2025)."""
    from ssla_b200.synthetic import event_batch

    gold = torch.load(GOLDEN / "model_mos_s_b8.pt")
    m = _model("S")
    ev, ln = event_batch(gold["batch"], seed=gold["seed"])
    from ssla_b200.model import async_event_to_grid, preprocess_inputs

    with torch.no_grad():
        x = preprocess_inputs(ev.cuda(), ln.cuda(), m.frame_size, m.hot_pixel_thres)
        taps = []
        for i, layer in enumerate(m.backbone):
            x = layer(x)
            if i in m.output_indices:
                taps.append(x)
        grids = [async_event_to_grid(t, m.grid_sizes[k], m.in_features[k]) for k, t in enumerate(taps)]
        for i, (a, b) in enumerate(zip(grids, gold["grids"])):
            assert_close(a, b, FP32_TOL, f"grid {i}")
        torch.backends.cudnn.allow_tf32 = False
        head = m.head(grids)
    assert_close(head, gold["head"], 1e-4, "head")


def test_layers_backward_runs():
    """Training path: gradients flow through routing, scan and gather-back."""
    m = _model("S").train()
    ev, ln = _events(1)
    out = m(ev, ln)
    out.square().mean().backward()
    g = m.backbone[1].scatter_conv_weights.grad
    assert g is not None and torch.isfinite(g).all() and g.abs().sum() > 0


@pytest.mark.parametrize("C", [1, 4, 7, 12, 24, 32, 48, 96, 128, 256])
def test_layernorm_residual_matches_torch(C):
    from ssla_b200.ops.mos import layernorm_residual

    gen = torch.Generator().manual_seed(C)
    x = torch.randn(5000, C, generator=gen).cuda()
    r = torch.randn(5000, C, generator=gen).cuda()
    w = torch.randn(C, generator=gen).cuda()
    b = torch.randn(C, generator=gen).cuda()
    ref = torch.nn.functional.layer_norm(x + r, (C,), w, b, 1e-5)
    assert rel_err(layernorm_residual(x, r, w, b, 1e-5), ref) < FP32_TOL
    assert rel_err(layernorm_residual(x, None, w, b, 1e-5),
                   torch.nn.functional.layer_norm(x, (C,), w, b, 1e-5)) < FP32_TOL


@pytest.mark.parametrize("k,I,C,scatter,gather", [(3, 12, 12, True, True), (3, 12, 24, True, True),
                                                   (1, 2, 12, True, True), (3, 24, 24, False, False)])
def test_mos_attention_fused_inference_matches_autograd_path(k, I, C, scatter, gather):
    """The no-grad path (q/v/g folded into the scatter weights, o into the gather weights, one
    fused gather + gate + scan kernel, fused residual LayerNorm) against the autograd path of
    the same layer on the same inputs."""
    from ssla_b200.layers import MosAttention
    from ssla_b200.model import preprocess_inputs
    from ssla_b200.synthetic import seeded_parameters

    ev, ln = _events(1)
    x = preprocess_inputs(ev, ln, (240, 304))
    x["events"] = torch.randn(x["events"].shape[0], I, generator=torch.Generator().manual_seed(1)).cuda()
    layer = MosAttention(I, C, (240, 304), [k, k], scatter_proj=scatter, gather_proj=gather)
    seeded_parameters(layer, 11)
    layer = layer.cuda()
    with torch.enable_grad():
        ref = layer(dict(x))["events"]
    with torch.no_grad():
        fused = layer(dict(x))["events"]
    assert rel_err(fused, ref.detach()) < FP32_TOL


@pytest.mark.parametrize("frame,k,stride", [((40, 52), 3, 1), ((40, 52), 2, 2), ((31, 17), 3, 1), ((30, 38), 4, 4),
                                            ((12, 12), 5, 1)])
def test_routing_kernels_match_torch_formulation(frame, k, stride):
    """GPU routing (pixel map + per-field merge) against the PyTorch formulation run on the CPU:
    identical fields, lengths, and (src, pos, time) order, with timestamp ties inside and across
    pixels, frame borders, and an empty sample."""
    from ssla_b200.utils.routing import replicate_to_fields

    gen = torch.Generator().manual_seed(frame[0] * 100 + k)
    B, (H, W) = 3, frame
    pix = torch.randperm(B * H * W, generator=gen)[: B * H * W // 5]
    pix = pix[pix // (H * W) != 1].sort().values  # sample 1 empty
    G = pix.numel()
    lengths = torch.randint(1, 6, (G,), generator=gen)
    times = torch.cat([torch.randint(0, 8, (int(n),), generator=gen).sort().values for n in lengths])
    bid, rem = pix // (H * W), pix % (H * W)
    args = (bid, rem // W, rem % W, lengths, times, frame, (k, k), (stride, stride))
    ref = replicate_to_fields(*args, batch_size=B)
    got = replicate_to_fields(*(a.cuda() if torch.is_tensor(a) else a for a in args), batch_size=B)
    for key in ("field_id", "lengths", "src", "pos_id", "time"):
        assert torch.equal(got[key].cpu(), ref[key]), key


def test_mos_attention_in_kernel_projection_matches(monkeypatch):
    """The memory-saving inference variant (projection inside the scan kernel) against the
    GEMM-fed one on the same layer and inputs."""
    import ssla_b200.ops.mos as mos
    from ssla_b200.layers import MosAttention
    from ssla_b200.model import preprocess_inputs
    from ssla_b200.synthetic import seeded_parameters

    ev, ln = _events(1)
    x = preprocess_inputs(ev, ln, (240, 304))
    x["events"] = torch.randn(x["events"].shape[0], 12, generator=torch.Generator().manual_seed(2)).cuda()
    layer = MosAttention(12, 24, (240, 304), [3, 3])
    seeded_parameters(layer, 5)
    layer = layer.cuda()
    with torch.no_grad():
        ref = layer(dict(x))["events"]
        monkeypatch.setattr(mos, "Y_BYTES_LIMIT", 0)
        got = layer(dict(x))["events"]
    assert rel_err(got, ref) < FP32_TOL


@pytest.mark.parametrize("M,K,N", [(4097, 12, 324), (3000, 108, 12), (513, 7, 45), (1000, 216, 24), (0, 12, 12)])
def test_matmul_rows_matches_torch(M, K, N):
    """The skinny fp32 row kernel (MoS inference projections) against a float64 product, on
    vectorised (K % 4 == 0) and scalar row paths, a strided A and an empty A."""
    from ssla_b200.ops.mos import matmul_rows

    gen = torch.Generator().manual_seed(M + K + N)
    a_full = torch.randn(M, K + 3, generator=gen)
    a = a_full[:, :K] if K % 4 else torch.randn(M, K, generator=gen)
    b = torch.randn(K, N, generator=gen)
    ref = (a.double() @ b.double()).float()
    got = matmul_rows(a.cuda(), b.cuda())
    assert got.shape == (M, N)
    if M:
        assert rel_err(got, ref) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,N", [(1, 4, 16), (300, 12, 324), (5000, 48, 1296), (4097, 864, 96), (70000, 36, 40),
                                   (3000, 96, 2592), (700, 24, 648), (5000, 12, 324), (4500, 8, 130),
                                   (130, 100, 130)])
def test_matmul_tc_split_tf32(M, K, N):
    """The split-TF32 tensor-core GEMM (csrc/gemm_tf32.cu) against a float64 product: partial
    tiles in M, N and K, N below and above one tile, K up to 864.  Bound: 2e-5 of the largest
    output magnitude (the fp32 cuBLAS product lands near 1e-6 here)."""
    from ssla_b200.ops.mos import RowsGemm, check_tc_errors, matmul_tc, split_tf32

    gen = torch.Generator().manual_seed(M + K + N)
    a = torch.randn(M, K, generator=gen)
    b = torch.randn(N, K, generator=gen) / K ** 0.5
    ref = a.double() @ b.double().t()
    got = matmul_tc(a.cuda(), split_tf32(b.cuda()))
    check_tc_errors("cuda")
    assert got.shape == (M, N)
    err = (got.cpu().double() - ref).abs().max() / ref.abs().max()
    assert err < 2e-5, float(err)
    rg = RowsGemm(b.t().cuda())  # dispatch: tensor cores from TC_MIN_ROWS rows, row kernel below
    assert ((rg(a.cuda()).cpu().double() - ref).abs().max() / ref.abs().max()) < 2e-5


@pytest.mark.parametrize("I,C", [(2, 12), (12, 12)])
def test_linear_attention_matches_reference(I, C):
    """LinearAttention (layers/linear_attention.py:39-102) against the reference layer's output
    on the same pixel groups and seeded weights (tests/golden/make_golden_model.py)."""
    from ssla_b200.layers import LinearAttention
    from ssla_b200.model import preprocess_inputs
    from ssla_b200.synthetic import event_batch, seeded_parameters

    gold = torch.load(GOLDEN / "linear_attention.pt")
    ev, ln = event_batch(1, seed=gold["seed"])
    x = preprocess_inputs(ev.cuda(), ln.cuda(), (240, 304))
    if I != 2:
        x["events"] = torch.randn(x["events"].shape[0], I, generator=torch.Generator().manual_seed(13)).cuda()
    layer = LinearAttention(I, C, (240, 304)).eval()
    seeded_parameters(layer, 500 + I)
    with torch.no_grad():
        out = layer.cuda()(x)["events"]
    assert rel_err(out, gold[f"in{I}_h{C}"]) < FP32_TOL


def _nms_reference(preds, C, frame, conf, iou, filtering, max_det):
    """The reference post-processing (model_mos.py:20-29, 232-299) on torchvision's nms."""
    from torchvision.ops import nms

    cx, cy, w, h = preds[..., :4].unbind(-1)
    boxes = torch.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], -1)
    obj = preds[..., 4].sigmoid()
    cc, cp = preds[..., 5:5 + C].sigmoid().max(-1)
    scores = obj * cc
    out = []
    for b in range(preds.shape[0]):
        bb, bs, bl = boxes[b], scores[b], cp[b].to(torch.int64)
        if filtering:
            k = bs >= conf
            bb, bs, bl = bb[k], bs[k], bl[k]
        keep = nms(bb + (bl * float(max(frame) + 1))[:, None], bs, iou)[:max_det]
        out.append((bb[keep], bs[keep], bl[keep]))
    return out


@pytest.mark.parametrize("N,filtering,max_det", [(1140, True, 100), (1140, False, 100), (300, True, 5), (3000, True, 300)])
def test_batched_nms_matches_torchvision(N, filtering, max_det):
    """GPU batched NMS against the reference post-processing on torchvision's nms (clustered
    boxes so many overlap, continuous scores so the order has no ties).  torchvision is a
    third-party library of the reference, used here only as the checker."""
    from ssla_b200.model import postprocess_with_nms

    gen = torch.Generator().manual_seed(N + max_det)
    B, C, frame = 6, 2, (240, 304)
    centers = torch.rand(B, 12, 2, generator=gen) * torch.tensor([304.0, 240.0])
    pick = torch.randint(0, 12, (B, N), generator=gen)
    cxy = torch.gather(centers, 1, pick[..., None].expand(B, N, 2)) + 6 * torch.randn(B, N, 2, generator=gen)
    wh = 20 + 30 * torch.rand(B, N, 2, generator=gen)
    logits = torch.randn(B, N, 1 + C, generator=gen) * 2 - 1
    preds = torch.cat([cxy, wh, logits], -1)
    # the checker runs on the same device so scores (sigmoid) are bit-identical on both sides
    ref = _nms_reference(preds.cuda(), C, frame, 0.2, 0.65, filtering, max_det)
    got = postprocess_with_nms(preds.cuda(), C, frame, 0.2, 0.65, filtering, max_det)
    for (rb, rs, rl), g in zip(ref, got):
        assert len(rl) > 0
        assert torch.equal(g["labels"], rl)
        assert torch.equal(g["scores"], rs)
        assert torch.equal(g["boxes"], rb)


@pytest.mark.parametrize("maxpp,keep", [(512, 50), (512, None), (3, None), (100, 7)])
def test_group_events_kernels_exact(maxpp, keep):
    """Native pixel grouping (csrc/group.cu) against the CPU restatement of the reference's
    stable-sort grouping (oracle.routing), on batches with hot pixels: one pixel with 40 events
    (the per-thread ranking path), one with 700 (shared-memory sort) and one with 5000 (radix
    selection of the kept ranks), plus an empty sample and duplicate timestamps."""
    from oracle import routing as orr
    from ssla_b200.synthetic import event_batch
    from ssla_b200.utils.routing import group_events

    ev, ln = event_batch(3, seed=5)
    ev, ln = ev.clone(), ln.clone()
    ln[1] = 0
    gen = torch.Generator().manual_seed(1)
    for cnt, (x, y) in ((40, (10, 20)), (700, (100, 50)), (5000, (303, 239))):
        idx = torch.randperm(int(ln[0]), generator=gen)[:cnt]
        ev[0, idx, 0], ev[0, idx, 1] = float(x), float(y)
    ev[2, 100:110, 2] = ev[2, 100, 2]  # equal timestamps
    x = torch.cat([ev[..., :3], ev[..., 2:3], ev[..., 3:]], dim=-1)
    ref = orr.group_events(x, ln, (240, 304), maxpp)
    if keep is not None:
        st = torch.cumsum(ref["lengths"], 0) - ref["lengths"]
        pos = torch.arange(ref["events"].shape[0]) - torch.repeat_interleave(st, ref["lengths"])
        k = pos < keep
        ref["events"], ref["time"] = ref["events"][k], ref["time"][k]
        ref["lengths"] = ref["lengths"].clamp(max=keep)
    got = group_events((x.cuda(), ln.cuda()), (240, 304), maxpp, keep_first=keep)
    for key in ("events", "time", "batch_id", "h", "w", "lengths"):
        assert torch.equal(got[key].cpu(), ref[key]), key


def test_preprocess_delay_matches_oracle():
    """Grouping + hot-pixel truncation + per-pixel delay in one pass (model.preprocess_inputs)
    against the reference's three-step preprocessing restated in oracle.routing.preprocess."""
    from oracle import routing as orr
    from ssla_b200.model import preprocess_inputs
    from ssla_b200.synthetic import event_batch

    ev, ln = event_batch(4, seed=9)
    ref = orr.preprocess(ev, ln, (240, 304), 50)
    got = preprocess_inputs(ev.cuda(), ln.cuda(), (240, 304), 50)
    for key in ("events", "time", "batch_id", "h", "w", "lengths"):
        assert torch.equal(got[key].cpu(), ref[key]), key


@pytest.mark.parametrize("P,Pg", [(9, 9), (9, 0), (1, 0), (1, 9)])
def test_patch_scan_routed_matches_indexed(P, Pg):
    """The patch scan with key / dst formed in the kernel from (src, pos) equals the scan over
    explicitly built index arrays, bit for bit."""
    from ssla_b200.ops import mos as _mos

    gen = torch.Generator().manual_seed(P * 10 + Pg)
    E, C, n = 5000, 12, 20000
    src = torch.randint(0, E, (n,), generator=gen)
    pos = torch.randint(0, P if P > 1 else 9, (n,), generator=gen)
    cuts = torch.randperm(n - 1, generator=gen)[:3000].sort().values + 1
    cu = torch.cat([torch.zeros(1, dtype=torch.int64), cuts, torch.tensor([n])])
    y = torch.randn(E * P, 3 * C, generator=gen)
    key = src * P + pos if P > 1 else src
    dst = src * Pg + pos if Pg > 0 else torch.arange(n)
    rows_out = E * Pg if Pg > 0 else n
    z_ref = torch.zeros(rows_out, C).cuda()
    z = torch.zeros(rows_out, C).cuda()
    if Pg > 0:  # (event, position) pairs must be unique for a deterministic result
        keep = torch.zeros(n, dtype=torch.bool)
        seen = set()
        for i, d in enumerate(dst.tolist()):
            if d not in seen:
                seen.add(d)
                keep[i] = True
        src, pos, key, dst = src[keep], pos[keep], key[keep], dst[keep]
        n = src.numel()
        cu = torch.unique(torch.clamp(cu, max=n))
    _mos.patch_scan(y.cuda(), key.cuda(), dst.cuda(), cu.cuda(), C, z_ref)
    _mos.patch_scan_routed(y.cuda(), src.cuda(), pos.cuda() if (P > 1 or Pg > 0) else None, P, Pg, cu.cuda(), C, z)
    assert torch.equal(z.cpu(), z_ref.cpu())
