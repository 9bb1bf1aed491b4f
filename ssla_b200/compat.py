"""Run the reference's own model code (model_mos.py and the modules it imports) on top of
ssla_b200.

The reference resolves its hot-path modules by top-level import paths (model_mos.py:11-17,
layers/*.py, utils/*.py).  ``alias_reference_modules()`` registers ssla_b200's implementations
under those names in ``sys.modules``, so that a later ``import model_mos`` (with the reference
sources on ``sys.path``) builds its layer stack from ssla_b200:

=============================  =========================================
reference import path          served by
=============================  =========================================
layers.mos_attention           ssla_b200.layers.mos_attention
layers.linear_attention        ssla_b200.layers.linear_attention
layers.sparse_pooling          ssla_b200.layers.sparse_pooling
layers.temporal_dropout        ssla_b200.layers.temporal_dropout
layers.async_sparse_module     ssla_b200.layers.async_sparse_module
utils.async_utils              ssla_b200.utils.async_utils
utils.farsecnn_utils           ssla_b200.utils.farsecnn_utils
ops.common.scan                ssla_b200.ops.common.scan
ops.gla.chunk                  ssla_b200.ops.gla.chunk
ops.gla.chunk_scalar           ssla_b200.ops.gla.chunk_scalar
ops.gla.fused_recurrent        ssla_b200.ops.gla.fused_recurrent
torch_scatter                  ssla_b200.torch_scatter
=============================  =========================================

Everything else (model_mos.py itself, model_base.py, layers/yolox_head.py, layers/mos_lstm.py,
utils/data_utils.py, the datasets) stays the reference's.  Call it before the first import of
any reference module.
"""
from __future__ import annotations

import importlib
import sys

ALIASES = {
    "layers.mos_attention": "ssla_b200.layers.mos_attention",
    "layers.linear_attention": "ssla_b200.layers.linear_attention",
    "layers.sparse_pooling": "ssla_b200.layers.sparse_pooling",
    "layers.temporal_dropout": "ssla_b200.layers.temporal_dropout",
    "layers.async_sparse_module": "ssla_b200.layers.async_sparse_module",
    "utils.async_utils": "ssla_b200.utils.async_utils",
    "utils.farsecnn_utils": "ssla_b200.utils.farsecnn_utils",
    "ops.common.scan": "ssla_b200.ops.common.scan",
    "ops.gla.chunk": "ssla_b200.ops.gla.chunk",
    "ops.gla.chunk_scalar": "ssla_b200.ops.gla.chunk_scalar",
    "ops.gla.fused_recurrent": "ssla_b200.ops.gla.fused_recurrent",
    "torch_scatter": "ssla_b200.torch_scatter",
}


def alias_reference_modules() -> dict:
    """Register the ssla_b200 modules under the reference's import paths; returns the mapping
    of reference name -> module."""
    done = {}
    for ref_name, ours in ALIASES.items():
        mod = importlib.import_module(ours)
        sys.modules[ref_name] = mod
        done[ref_name] = mod
    return done
