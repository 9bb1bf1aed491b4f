"""The reference's own model_mos.py, unchanged, running on top of ssla_b200.

``ssla_b200.compat.alias_reference_modules()`` serves the reference's hot-path import paths
(layers.mos_attention, layers.sparse_pooling, layers.temporal_dropout, utils.async_utils,
utils.farsecnn_utils, ops.common.scan, torch_scatter, ...) from ssla_b200; the reference's
MosModel (model_mos.py:125-170), its preprocessing, grid densification and YOLOX head
(layers/yolox_head.py) are imported from the installed reference (baseline/_ref, made by
baseline/install_ref.sh) and run on the GPU.  Test-side stubs cover only the training and
evaluation dependencies the model file imports (lightning, pycocotools, h5py, hdf5plugin).
The result is compared with the fixture the reference produced on the CPU
(tests/golden/make_golden_model.py: batch 2, event_batch seed 7, weights seed 2025)."""
import subprocess
import sys
import textwrap

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu
REF = ROOT / "baseline" / "_ref"

SCRIPT = textwrap.dedent(r'''
    import sys, types
    import torch, yaml
    sys.path.insert(0, "{root}")

    def stub(name, **attrs):
        m = types.ModuleType(name)
        m.__dict__.update(attrs)
        sys.modules[name] = m

    class LightningModule(torch.nn.Module):
        pass

    for n in ("lightning", "lightning.pytorch", "lightning.pytorch.core", "pycocotools", "h5py", "hdf5plugin"):
        stub(n)
    stub("lightning.pytorch.core.module", LightningModule=LightningModule)
    stub("lightning.pytorch.utilities", grad_norm=lambda *a, **k: {{}})
    stub("pycocotools.coco", COCO=object)
    stub("pycocotools.cocoeval", COCOeval=object)

    from ssla_b200.compat import alias_reference_modules
    aliased = alias_reference_modules()
    sys.path.insert(0, "{ref}")
    import model_mos                                   # the reference file, unchanged
    import layers.mos_attention, layers.sparse_pooling, layers.temporal_dropout
    assert model_mos.MosAttention.__module__ == "ssla_b200.layers.mos_attention", model_mos.MosAttention.__module__
    assert model_mos.SparseMaxPool.__module__ == "ssla_b200.layers.sparse_pooling"
    assert model_mos.TemporalDropout.__module__ == "ssla_b200.layers.temporal_dropout"
    assert model_mos.group_events.__module__.startswith("ssla_b200.")
    assert model_mos.YOLOXHead.__module__ == "layers.yolox_head"  # the reference's own head

    from ssla_b200.synthetic import event_batch, seeded_parameters
    gold = torch.load("{gold}")
    cfg = yaml.safe_load(open("{ref}/ssla_configs/model/MOS_S.yaml"))
    model = model_mos.MosModel(cfg, hot_pixel_thres=50, dataset="Gen1")
    seeded_parameters(model, gold["param_seed"])
    model = model.cuda().eval()
    events, lengths = event_batch(gold["batch"], seed=gold["seed"])
    labels = torch.tensor([[[100.0, 100.0, 40.0, 30.0, 0.0]], [[150.0, 80.0, 50.0, 40.0, 1.0]]])[: gold["batch"]]
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    with torch.no_grad():
        out = model(dict(events=events.cuda(), lengths=lengths.cuda(), labels=labels.cuda()))
    head = out["output"].cpu().double()
    ref = gold["head"].double()
    rms = float((head - ref).norm() / ref.norm())
    mx = float((head - ref).abs().max() / ref.abs().max())
    print("RESULT", rms, mx, tuple(head.shape))
''')


def test_reference_model_mos_runs_unchanged_on_ssla_b200(tmp_path):
    if not (REF / "model_mos.py").exists():
        pytest.skip("reference not installed into baseline/_ref (bash baseline/install_ref.sh)")
    script = tmp_path / "run_ref_model.py"
    script.write_text(SCRIPT.format(root=ROOT, ref=REF, gold=ROOT / "tests" / "golden" / "model_mos_s.pt"))
    # a fresh interpreter: the reference's top-level package names (layers, utils, ops) must not
    # clash with modules other tests imported
    r = subprocess.run([sys.executable, str(script)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("RESULT")][-1].split()
    rms, mx = float(line[1]), float(line[2])
    # the head decode exponentiates box sizes: 1e-4 relative for the dense head (as the
    # ssla_b200 runner's own full-model test)
    assert rms < 1e-4 and mx < 5e-4, (rms, mx)
