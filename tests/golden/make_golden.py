"""Generate the golden fixtures in this folder from the reference implementation itself.

Run in a container that has the haohq19/ssla sources (read-only) and no GPU:

    python tests/golden/make_golden.py /path/to/ssla

It imports the reference package and runs
  * its naive PyTorch forms (ops/gla/naive.py, ops/gla/naive_scalar.py), and
  * its Triton kernels (ops/gla/chunk.py ``chunk_gla`` fwd+bwd, ops/common/scan.py ``scan``
    fwd+bwd) under the Triton CPU interpreter,
on small seeded inputs, and saves inputs and outputs as ``*.pt``.  Harness-side shims only,
the reference sources are not modified:
  * ``TRITON_INTERPRET=1``; ``triton.autotune`` pinned to its first config (the autotuner
    needs a GPU driver);
  * ``ops.utils.op.exp`` re-bound to a jitted ``tl.exp`` wrapper (the module-level alias
    escapes the interpreter's patching);
  * ``torch.cpu.device`` made a no-op context (``input_guard`` enters it for CPU tensors).
The tests (tests/test_oracle.py) check the ``oracle`` package against these files.
"""
from __future__ import annotations

import contextlib
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402

OUT = Path(__file__).resolve().parent


def _install_shims():
    def autotune(configs, key=None, **kw):
        cfg = configs[0]

        def deco(fn):
            class Pinned(triton.runtime.KernelInterface):
                def __init__(self, fn):
                    self.fn = fn
                    self.arg_names = fn.arg_names

                def __getattr__(self, name):
                    return getattr(self.fn, name)

                def run(self, *args, **kwargs):
                    kwargs = {**cfg.kwargs, **kwargs, "num_warps": cfg.num_warps}
                    return self.fn.run(*args, **kwargs)

            return Pinned(fn)

        return deco

    triton.autotune = autotune
    torch.cpu.device = lambda *a, **k: contextlib.nullcontext()


def main(ref_root: str):
    _install_shims()
    sys.path.insert(0, ref_root)
    import ops.utils.op as op_mod

    @triton.jit
    def _exp(x):
        return tl.exp(x)

    op_mod.exp = _exp
    import ops.gla.chunk as chunk_mod
    import ops.common.chunk_h as chunk_h_mod
    chunk_mod.exp = _exp
    chunk_h_mod.exp = _exp
    from ops.gla.naive import naive_gla_recurrent, naive_gla_parallel
    from ops.gla.naive_scalar import naive_gla_recurrent_scalar
    from ops.gla.chunk import chunk_gla
    from ops.common.scan import scan

    # ---- c1 anchor: B=2, H=4, T=64, K=V=32, fp32, seed 0
    torch.manual_seed(0)
    B, H, T, K, V = 2, 4, 64, 32, 32
    q = torch.randn(B, H, T, K)
    k = torch.randn(B, H, T, K) * K ** -0.5
    v = torch.randn(B, H, T, V)
    gk = F.logsigmoid(torch.randn(B, H, T, K)) / 16
    cv = lambda x: x.permute(0, 2, 1, 3).reshape(B * T, H, -1).contiguous()
    q, k, v, gk = map(cv, (q, k, v, gk))
    cu = torch.arange(B + 1) * T
    o, ht = naive_gla_recurrent(q, k, v, gk, cu, output_final_state=True)
    op = naive_gla_parallel(q, k, v, gk, cu)
    torch.save(dict(q=q, k=k, v=v, g=gk, cu=cu, o=o, ht=ht, o_parallel=op), OUT / "c1_naive_recurrent.pt")
    print("c1", float(o.sum()), float(o.norm()), float(ht.sum()), float(ht.norm()))

    # ---- chunk_gla fwd+bwd under the interpreter: varlen [20, 44], H=2, K=V=32, with h0
    torch.manual_seed(1)
    T, H, K, V = 64, 2, 32, 32
    cu = torch.tensor([0, 20, 64])
    q = torch.randn(T, H, K, requires_grad=True)
    k = (torch.randn(T, H, K) * K ** -0.5).requires_grad_()
    v = torch.randn(T, H, V, requires_grad=True)
    g = (F.logsigmoid(torch.randn(T, H, K)) / 16).requires_grad_()
    h0 = (torch.randn(2, H, K, V) * 0.1).requires_grad_()
    do = torch.randn(T, H, V)
    dht = torch.randn(2, H, K, V)
    o, ht = chunk_gla(q, k, v, g, cu, initial_state=h0, output_final_state=True)
    (o * do).sum().add_((ht * dht).sum()).backward()
    torch.save(dict(q=q.detach(), k=k.detach(), v=v.detach(), g=g.detach(), h0=h0.detach(), cu=cu,
                    do=do, dht=dht, o=o.detach(), ht=ht.detach(), dq=q.grad, dk=k.grad, dv=v.grad,
                    dg=g.grad, dh0=h0.grad), OUT / "chunk_gla_interp.pt")
    print("chunk_gla", float(o.sum()))

    # ---- scan fwd+bwd under the interpreter: T=64, C=8, three sequences
    torch.manual_seed(2)
    T, C = 64, 8
    cu = torch.tensor([0, T // 3, 2 * (T // 3), T])
    u = torch.randn(T, C, requires_grad=True)
    gs = torch.exp(F.logsigmoid(torch.randn(T, C))).requires_grad_()
    h = scan(u, gs, cu)
    dh = torch.randn(T, C)
    (h * dh).sum().backward()
    torch.save(dict(u=u.detach(), g=gs.detach(), cu=cu, h=h.detach(), dh=dh, du=u.grad, dg=gs.grad),
               OUT / "scan_interp.pt")
    print("scan", float(h.sum()))

    # ---- scalar GLA naive form
    torch.manual_seed(3)
    T, H = 50, 6
    cu = torch.tensor([0, 7, 30, 50])
    qs, ks, vs = torch.randn(T, H), torch.randn(T, H), torch.randn(T, H)
    gss = F.logsigmoid(torch.randn(T, H))
    h0s = torch.randn(3, H)
    os_, hts = naive_gla_recurrent_scalar(qs, ks, vs, gss, cu, initial_state=h0s, output_final_state=True)
    torch.save(dict(q=qs, k=ks, v=vs, g=gss, cu=cu, h0=h0s, o=os_, ht=hts), OUT / "gla_scalar_naive.pt")
    print("scalar", float(os_.sum()))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path to the ssla sources>")
    main(sys.argv[1])
