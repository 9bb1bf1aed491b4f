"""SSLA model runner on the ssla_b200 layers: event preprocessing, the layer stack built from a
model config (the dict of configs/model/MOS_*.yaml), dense grids from the last event of every
output cell, and the YOLOX detection head's inference decode.

Mirrors model_mos.py:32-228 (get_module, get_modulelist, MosModel.forward / preprocess_inputs /
async_event_to_grid) and the forward / decode of layers/yolox_head.py:96-258, with the same
module and parameter names, so reference checkpoints load.  Training-only parts of the
reference (SimOTA assignment and losses, Lightning hooks, COCO evaluation) are not part of this
runner.
"""
from __future__ import annotations

import math
from typing import Dict, List

import torch
import torch.nn as nn

from .layers import (LinearAttention, MosAttention, SparseAdaptiveAvgPool, SparseAdaptiveMaxPool, SparseAvgPool,
                     SparseMaxPool, TemporalDropout)
from . import _lib
from .ops import segment as _seg
from .ops.mos import check_tc_errors
from .utils.farsecnn_utils import group_events

FRAME_SIZES = {"Gen1": ((240, 304), 2), "NCaltech101": ((180, 240), 101)}


def get_module(cfg: Dict, frame_size, channel_size: int) -> nn.Module:
    """One layer from its config entry (model_mos.py:32-86)."""
    name = cfg["name"]
    if name == "SparseMaxPool":
        return SparseMaxPool(frame_size, kernel_size=[cfg["kernel_size"]] * 2)
    if name == "SparseAvgPool":
        return SparseAvgPool(frame_size, kernel_size=[cfg["kernel_size"]] * 2)
    if name == "SparseAdaptiveMaxPool":
        return SparseAdaptiveMaxPool(frame_size, [cfg["output_size"]] * 2)
    if name == "SparseAdaptiveAvgPool":
        return SparseAdaptiveAvgPool(frame_size, [cfg["output_size"]] * 2)
    if name == "TemporalDropout":
        return TemporalDropout(cfg["window_size"], frame_size)
    if name == "MosAttention":
        k = cfg["kernel_size"]
        return MosAttention(input_size=channel_size, hidden_size=cfg["hidden_size"], frame_size=frame_size,
                            kernel_size=[min(k, frame_size[0]), min(k, frame_size[1])],
                            scatter_proj=cfg.get("scatter_proj", True), gather_proj=cfg.get("gather_proj", True))
    if name == "LinearAttention":
        return LinearAttention(input_size=channel_size, hidden_size=cfg["hidden_size"], frame_size=frame_size)
    raise ValueError("Module does not exist: ", name)


def get_modulelist(config_layers, sensor_size, in_channels, expected_strides):
    """Layer stack and its output taps (model_mos.py:89-122)."""
    layers, strides, feature_sizes, grid_sizes, output_indices = [], [], [], [], []
    grid_size, channel_size, stride = sensor_size, in_channels, 1
    for i, cfg in enumerate(config_layers):
        if cfg["name"] in ("SparseMaxPool", "SparseAvgPool"):
            if stride in expected_strides:
                strides.append(stride)
                feature_sizes.append(channel_size)
                grid_sizes.append(grid_size)
                output_indices.append(i)
            stride *= cfg["kernel_size"]
        m = get_module(cfg, grid_size, channel_size)
        layers.append(m)
        grid_size = m.frame_output_size
        channel_size = getattr(m, "hidden_size", channel_size)
    if stride in expected_strides and stride not in strides:
        strides.append(stride)
        feature_sizes.append(channel_size)
        grid_sizes.append(grid_size)
        output_indices.append(len(layers) - 1)
    return nn.ModuleList(layers), strides, feature_sizes, grid_sizes, output_indices


def preprocess_inputs(events: torch.Tensor, lengths: torch.Tensor, frame_size, hot_pixel_thres: int = 50):
    """<x, y, t, p> events -> pixel groups with per-event features <dt, p> (model_mos.py:173-209):
    dt = time since the previous event of the pixel / 1e5, clamped to 1, 1 for the first event;
    with hot_pixel_thres > 0 only the first `hot_pixel_thres` events of a pixel are kept (the
    reference truncates after computing dt; a pixel's kept events are a prefix of its grouped
    events, so truncating during the grouping gives the same dt)."""
    with torch.no_grad():
        x = torch.cat([events[..., :3], events[..., 2:3], events[..., 3:]], dim=-1)
        return group_events((x, lengths), frame_size, keep_first=hot_pixel_thres if hot_pixel_thres > 0 else None,
                            delay_col=0)


def async_event_to_grid(x, grid_size, channels: int) -> torch.Tensor:
    """Dense (B, C, Hg, Wg) grid holding the last event of every occupied cell
    (model_mos.py:212-228)."""
    last = torch.cumsum(x["lengths"], 0) - 1
    ev = x["events"][last]
    Hg, Wg = grid_size
    cell = x["batch_id"] * (Hg * Wg) + x["h"] * Wg + x["w"]
    B = x["batch_size"]
    grid = _seg.index_add_rows_ad(ev.float(), cell, B * Hg * Wg)
    return grid.reshape(B, Hg, Wg, channels).permute(0, 3, 1, 2)


class YOLOXHead(nn.Module):
    """Inference part of the YOLOX head (layers/yolox_head.py:96-258): 1x1 conv stems and
    predictors per level, decoded to (B, anchors, 4 + 1 + num_classes) boxes
    (cx, cy, w, h in pixels; objectness and class logits)."""

    def __init__(self, num_classes, strides, in_channels, width):
        super().__init__()
        self.num_classes = num_classes
        self.strides = strides
        self.cls_convs, self.reg_convs = nn.ModuleList(), nn.ModuleList()
        self.cls_preds, self.reg_preds, self.obj_preds = nn.ModuleList(), nn.ModuleList(), nn.ModuleList()
        stem = lambda c: nn.Sequential(nn.Conv2d(c, width, kernel_size=1), nn.BatchNorm2d(width), nn.SiLU())
        for c in in_channels:
            self.cls_convs.append(stem(c))
            self.reg_convs.append(stem(c))
            self.cls_preds.append(nn.Conv2d(width, num_classes, 1))
            self.reg_preds.append(nn.Conv2d(width, 4, 1))
            self.obj_preds.append(nn.Conv2d(width, 1, 1))
        prior = -math.log((1 - 0.01) / 0.01)
        with torch.no_grad():
            for m in list(self.cls_preds) + list(self.obj_preds):
                m.bias.fill_(prior)

    def forward(self, xin: List[torch.Tensor]) -> torch.Tensor:
        outs = []
        for k, x in enumerate(xin):
            cf = self.cls_convs[k](x)
            rf = self.reg_convs[k](x)
            o = torch.cat([self.reg_preds[k](rf), self.obj_preds[k](rf), self.cls_preds[k](cf)], 1)
            B, C, Hh, Ww = o.shape
            o = o.permute(0, 2, 3, 1).reshape(B, Hh * Ww, C).clone()
            yv, xv = torch.meshgrid(torch.arange(Hh, device=o.device), torch.arange(Ww, device=o.device),
                                    indexing="ij")
            grid = torch.stack((xv, yv), 2).reshape(1, Hh * Ww, 2).to(o.dtype)
            s = self.strides[k]
            o[..., :2] = (o[..., :2] + grid) * s
            o[..., 2:4] = torch.exp(o[..., 2:4]) * s
            outs.append(o)
        return torch.cat(outs, 1)


@torch.no_grad()
def postprocess_with_nms(preds: torch.Tensor, num_classes: int, frame_size, conf_thres: float = 0.001,
                         iou_thres: float = 0.65, filtering: bool = True, max_det: int = 100) -> List[Dict]:
    """Detections per image (model_mos.py:232-299): boxes xyxy, score = sigmoid(obj) *
    max(sigmoid(cls)), labels; candidates below ``conf_thres`` dropped (``filtering``), greedy
    NMS per class (class-offset boxes, model_mos.py:20-29) at ``iou_thres`` on the GPU
    (``ssla_batched_nms``), at most ``max_det`` per image, in score order."""
    if preds.dim() != 3 or preds.size(-1) < 6:
        raise ValueError("preds must be (B, N, 4 + 1 + C)")
    B, N, _ = preds.shape
    cx, cy, w, h = preds[..., :4].unbind(dim=-1)
    boxes = torch.stack([cx - 0.5 * w, cy - 0.5 * h, cx + 0.5 * w, cy + 0.5 * h], dim=-1)
    obj = preds[..., 4].sigmoid()
    class_conf, class_pred = preds[..., 5:5 + num_classes].sigmoid().max(dim=-1)
    scores = obj * class_conf
    labels = class_pred.to(torch.int64)
    max_dim = max(int(frame_size[0]), int(frame_size[1]))
    shifted = (boxes + (labels * float(max_dim + 1))[..., None]).float().contiguous()
    _lib.require_cuda(shifted, what="postprocess_with_nms")
    L = _lib.load()
    keep = torch.empty((B, max_det), device=preds.device, dtype=torch.int64)
    count = torch.empty(B, device=preds.device, dtype=torch.int64)
    nb = L.ssla_batched_nms_workspace_bytes(B)
    ws = torch.empty(max(nb, 1), device=preds.device, dtype=torch.uint8)
    sc = scores.float().contiguous()
    _lib.check(L.ssla_batched_nms(shifted.data_ptr(), sc.data_ptr(), B, N, int(filtering), float(conf_thres),
                                  float(iou_thres), max_det, keep.data_ptr(), count.data_ptr(), ws.data_ptr(), nb,
                                  _lib.stream_of(shifted)), "postprocess_with_nms")
    out = []
    for b, n in enumerate(count.tolist()):
        idx = keep[b, :n]
        out.append({"boxes": boxes[b][idx], "scores": scores[b][idx], "labels": labels[b][idx]})
    return out


class MosDetector(nn.Module):
    """Preprocessing + layer stack + grids + head (MosModel.forward, model_mos.py:157-170)."""

    def __init__(self, model_config: Dict, dataset: str = "Gen1", hot_pixel_thres: int = 50):
        super().__init__()
        self.frame_size, self.num_classes = FRAME_SIZES[dataset]
        self.hot_pixel_thres = hot_pixel_thres
        self.backbone, strides, feats, grids, outs = get_modulelist(
            model_config["layers"], self.frame_size, 2, model_config.get("expected_strides", [8, 16]))
        self.strides, self.in_features, self.grid_sizes, self.output_indices = strides, feats, grids, outs
        self.head = YOLOXHead(self.num_classes, strides, feats, feats[-1])

    def backbone_grids(self, events: torch.Tensor, lengths: torch.Tensor) -> List[torch.Tensor]:
        x = preprocess_inputs(events, lengths, self.frame_size, self.hot_pixel_thres)
        taps = []
        for i, layer in enumerate(self.backbone):
            x = layer(x)
            if i in self.output_indices:
                taps.append(x)
        return [async_event_to_grid(t, self.grid_sizes[k], self.in_features[k]) for k, t in enumerate(taps)]

    def forward(self, events: torch.Tensor, lengths: torch.Tensor, check_errors: bool = True) -> torch.Tensor:
        """Head output (B, anchors, 4 + 1 + num_classes).  With ``check_errors`` the device flag of
        the tensor-core GEMMs' bounded waits is read once at the end (one host synchronisation)
        and a timeout raises instead of returning untrustworthy detections."""
        out = self.head(self.backbone_grids(events, lengths))
        if check_errors:
            check_tc_errors(out.device)
        return out

    def postprocess_with_nms(self, preds: torch.Tensor, conf_thres: float = 0.001, iou_thres: float = 0.65,
                             filtering: bool = True, max_det: int = 100) -> List[Dict]:
        return postprocess_with_nms(preds, self.num_classes, self.frame_size, conf_thres, iou_thres, filtering,
                                    max_det)
