"""CPU oracle for the ssla_b200 parity tests — TEST INFRASTRUCTURE ONLY.

Plain PyTorch-on-CPU restatements of the reference algorithms of haohq19/ssla's
gated-linear-attention hot path.  Each function cites the reference file:line it follows.
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` may
import this package, and only as the checker / reported CPU baseline; the ssla_b200 product
path never calls it.

Pinning: the restatements are checked against golden vectors produced by the reference's own
code (``tests/golden/make_golden.py`` imports the reference and runs its naive PyTorch forms
and its Triton kernels under the Triton CPU interpreter); see ``tests/test_oracle.py``.
``oracle.routing`` restates the pixel grouping of utils/farsecnn_utils.py:130-174 and the model
preprocessing of model_mos.py:173-209; it is pinned against the reference model's own grouped
output (tests/golden/model_mos_s.pt, tests/test_oracle.py).
``torch_scatter`` is not installed anywhere in this environment, so the segment-reduction
oracle (``oracle.segment``) restates its documented semantics: parity unpinned for
torch_scatter itself.
"""
