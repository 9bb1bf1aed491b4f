"""Golden fixtures for the routing, layer and full-model parity tests, produced by the reference
implementation itself on the CPU.

    python tests/golden/make_golden_model.py /path/to/ssla

Harness-side shims only (the reference sources are not modified):
  * stub modules for the training/evaluation dependencies the model file imports
    (lightning, pycocotools, h5py, hdf5plugin);
  * ``torch_scatter`` (not installed; version unpinned by the reference) provided by the
    restated semantics in ``oracle.segment``;
  * ``ops.common.scan.scan`` replaced by ``oracle.gla.scan_ref_vectorized``, which matches the
    reference's Triton scan bit for bit (tests/test_oracle.py) and avoids running the kernel
    under the slow Triton interpreter;
  * ``torch.sort`` forced to ``stable=True``.  The reference orders each patch's events by an
    unstable sort on time (utils/async_utils.py:221, utils/farsecnn_utils.py:246); on its GPU
    platform that is CUDA's radix sort, which keeps equal keys in input order, while the CPU sort
    does not.  Stable sorting reproduces the GPU order on the CPU (equal timestamps inside one
    patch occur at the coarse levels of the model).
Input events come from ``ssla_b200.synthetic.event_batch`` (seeded) and weights from
``ssla_b200.synthetic.seeded_parameters`` (seeded, by parameter name), so neither is stored.
"""
from __future__ import annotations

import sys
import types
from pathlib import Path

import torch
import yaml

OUT = Path(__file__).resolve().parent
ROOT = OUT.parent.parent
sys.path.insert(0, str(ROOT))

from oracle import gla as og  # noqa: E402
from oracle import segment as oseg  # noqa: E402
from ssla_b200.synthetic import event_batch, seeded_parameters  # noqa: E402


def _stub(name, **attrs):
    m = types.ModuleType(name)
    for k, v in attrs.items():
        setattr(m, k, v)
    sys.modules[name] = m
    return m


def install_shims():
    class LightningModule(torch.nn.Module):
        pass

    _stub("lightning")
    _stub("lightning.pytorch")
    _stub("lightning.pytorch.core")
    _stub("lightning.pytorch.core.module", LightningModule=LightningModule)
    _stub("lightning.pytorch.utilities", grad_norm=lambda *a, **k: {})
    _stub("pycocotools")
    _stub("pycocotools.coco", COCO=object)
    _stub("pycocotools.cocoeval", COCOeval=object)
    _stub("h5py")
    _stub("hdf5plugin")

    def scatter_max(src, index, dim=-1, dim_size=None):
        idx = index[:, 0] if index.dim() == 2 else index
        return oseg.scatter_max(src, idx, int(dim_size))

    def scatter_mean(src, index, dim=-1, dim_size=None):
        idx = index[:, 0] if index.dim() == 2 else index
        return oseg.scatter_mean(src, idx, int(dim_size))

    _stub("torch_scatter", scatter_max=scatter_max, scatter_mean=scatter_mean)


def linear_attention(ref_root: str):
    """Reference LinearAttention (layers/linear_attention.py:39-102) on one synthetic sample's
    pixel groups: (input 2 -> hidden 12, with input / residual projections) and (12 -> 12, on
    seeded N(0,1) features).  Saved: the output events of both layers."""
    import layers.linear_attention as lin_mod
    from model_mos import MosModel  # noqa: F401  (imports the layer stack and its stubs)

    torch.set_grad_enabled(False)
    events, lengths = event_batch(1, seed=11)
    model = MosModel(yaml.safe_load(open(Path(ref_root) / "configs" / "model" / "MOS_S.yaml")), hot_pixel_thres=50,
                     dataset="Gen1")
    x = model.preprocess_inputs(events.clone(), lengths.clone())
    out = {}
    for I, C in ((2, 12), (12, 12)):
        layer = lin_mod.LinearAttention(I, C, (240, 304)).eval()
        seeded_parameters(layer, 500 + I)
        xi = dict(x)
        if I != 2:
            xi["events"] = torch.randn(x["events"].shape[0], I, generator=torch.Generator().manual_seed(13))
        out[f"in{I}_h{C}"] = layer(xi)["events"].clone()
    torch.save(dict(seed=11, **out), OUT / "linear_attention.pt")
    print("linear attention", {k: tuple(v.shape) for k, v in out.items()})


def main(ref_root: str):
    install_shims()
    _sort = torch.sort

    def stable_sort(input, dim=-1, descending=False, stable=True, *, out=None):
        return _sort(input, dim=dim, descending=descending, stable=True)

    torch.sort = stable_sort
    sys.path.insert(0, ref_root)
    import yaml
    import ops.common.scan as scan_mod

    scan_mod.scan = lambda u, g, cu_seqlens: og.scan_ref_vectorized(u, g, cu_seqlens)
    import layers.mos_attention as mos_mod
    import layers.linear_attention as lin_mod

    mos_mod.scan = scan_mod.scan
    lin_mod.scan = scan_mod.scan
    from model_mos import MosModel
    from utils.async_utils import scatter_group_events_to_patch
    from utils.farsecnn_utils import gather_receptive_fields, compute_rf2pixels

    torch.set_grad_enabled(False)
    for variant, B in (("S", 2), ("L", 1)):
        events, lengths = event_batch(B, seed=7)
        cfg = yaml.safe_load(open(Path(ref_root) / "configs" / "model" / f"MOS_{variant}.yaml"))
        model = MosModel(cfg, hot_pixel_thres=50, dataset="Gen1").eval()
        seeded_parameters(model, 2025)
        x = model.preprocess_inputs(events.clone(), lengths.clone())
        g0 = {k: (v.clone() if torch.is_tensor(v) else v) for k, v in x.items()}
        taps, per_layer = [], {}
        for i, layer in enumerate(model.backbone):
            xin = {k: (v.clone() if torch.is_tensor(v) else v) for k, v in x.items()}
            if variant == "S" and i == 1:
                # routing of a 3x3 MoS layer and of the following 2x2 pooling, on this layer's input
                p = scatter_group_events_to_patch(xin, frame_size=layer.frame_size, patch2pixel_lut=layer.patch2pixel_lut)
                per_layer["patch"] = {"orig_event_idx": p["orig_event_idx"].to(torch.int32),
                                      "pos_id": p["pos_id"].to(torch.int8),
                                      "lengths": p["lengths"].to(torch.int32)}
            x = layer(x)
            if variant == "S" and i in (1, 3):
                per_layer[f"layer{i}"] = {"events": x["events"].clone(), "time": x["time"].to(torch.int32),
                                          "lengths": x["lengths"].to(torch.int32)}
            if variant == "S" and i == 1:
                lut, oc = compute_rf2pixels(layer.frame_size, (2, 2), (2, 2))
                xx = {k: (v.clone() if torch.is_tensor(v) else v) for k, v in x.items()}
                rf = gather_receptive_fields(xx, layer.frame_size, lut, oc)
                per_layer["rf2x2"] = {k: (v.to(torch.int32) if k != "events" else v) for k, v in rf.items()
                                      if torch.is_tensor(v)}
            if i in model.output_indices:
                taps.append(x)
        grids = [model.async_event_to_grid(t, k).float() for k, t in enumerate(taps)]
        labels = torch.tensor([[[100.0, 100.0, 40.0, 30.0, 0.0]], [[150.0, 80.0, 50.0, 40.0, 1.0]]])[:B]
        head_out = model.head(grids, labels)["output"]
        grouped = {k: (g0[k] if k == "events" else g0[k].to(torch.int32))
                   for k in ("events", "time", "lengths", "h", "w", "batch_id")}
        torch.save(dict(batch=B, seed=7, param_seed=2025, grouped=grouped if variant == "S" else None,
                        grids=grids, head=head_out, **per_layer), OUT / f"model_mos_{variant.lower()}.pt")
        print(variant, [g.shape for g in grids], float(grids[0].abs().sum()), head_out.shape)


def batch8(ref_root: str):
    """SSLA-S (MOS_S) forward at batch 8 (BASELINE config 5 with 8 samples, the per-GPU share
    of the batch of 64 on 8 GPUs): backbone grids and head output of the reference model.
    Same shims as ``main``; inputs ``event_batch(8, seed=21)``, weights ``seeded_parameters``
    with seed 2025."""
    import yaml
    import ops.common.scan as scan_mod
    import layers.mos_attention as mos_mod
    import layers.linear_attention as lin_mod

    scan_mod.scan = lambda u, g, cu_seqlens: og.scan_ref_vectorized(u, g, cu_seqlens)
    mos_mod.scan = scan_mod.scan
    lin_mod.scan = scan_mod.scan
    from model_mos import MosModel

    torch.set_grad_enabled(False)
    B = 8
    events, lengths = event_batch(B, seed=21)
    cfg = yaml.safe_load(open(Path(ref_root) / "configs" / "model" / "MOS_S.yaml"))
    model = MosModel(cfg, hot_pixel_thres=50, dataset="Gen1").eval()
    seeded_parameters(model, 2025)
    x = model.preprocess_inputs(events.clone(), lengths.clone())
    taps = []
    for i, layer in enumerate(model.backbone):
        x = layer(x)
        if i in model.output_indices:
            taps.append(x)
    grids = [model.async_event_to_grid(t, k).float() for k, t in enumerate(taps)]
    # the head also computes its training losses, so it needs labels: one box per sample
    labels = torch.tensor([[[60.0 + 20 * b, 50.0 + 15 * b, 40.0, 30.0, float(b % 2)]] for b in range(B)])
    head_out = model.head(grids, labels)["output"]
    torch.save(dict(batch=B, seed=21, param_seed=2025, grids=grids, head=head_out), OUT / "model_mos_s_b8.pt")
    print("S batch 8", [g.shape for g in grids], head_out.shape)


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3):
        sys.exit("usage: make_golden_model.py <path to the ssla sources> [--linear-attention-only | --batch8]")
    if len(sys.argv) == 3 and sys.argv[2] == "--batch8":
        install_shims()
        _sort = torch.sort
        torch.sort = lambda input, dim=-1, descending=False, stable=True, *, out=None: _sort(
            input, dim=dim, descending=descending, stable=True)
        sys.path.insert(0, sys.argv[1])
        batch8(sys.argv[1])
    elif len(sys.argv) == 3:
        install_shims()
        _sort = torch.sort
        torch.sort = lambda input, dim=-1, descending=False, stable=True, *, out=None: _sort(
            input, dim=dim, descending=descending, stable=True)
        sys.path.insert(0, sys.argv[1])
        import yaml  # noqa: F401
        import ops.common.scan as scan_mod
        import layers.linear_attention as lin_mod

        scan_mod.scan = lambda u, g, cu_seqlens: og.scan_ref_vectorized(u, g, cu_seqlens)
        lin_mod.scan = scan_mod.scan
        linear_attention(sys.argv[1])
    else:
        main(sys.argv[1])
