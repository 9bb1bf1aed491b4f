"""CPU checks of the C-ABI boundary: the library loads, exports every symbol declared in
include/ssla_b200.h, and the Python mirror raises the reference's exception types before
any kernel would run."""
import re

import pytest
import torch

from conftest import ROOT


def _declared():
    txt = (ROOT / "include" / "ssla_b200.h").read_text()
    return sorted(set(re.findall(r"^\w[\w\s\*]*?\b(ssla_\w+)\s*\(", txt, flags=re.M)))


def test_header_declares_entry_points():
    names = _declared()
    assert "ssla_chunk_gla_fwd" in names and "ssla_scan_fwd" in names
    assert len(names) >= 18


def test_library_exports_every_declared_symbol():
    from ssla_b200 import _lib

    lib = _lib.load()
    for n in _declared():
        assert hasattr(lib, n), n
    assert set(_declared()) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"
    assert lib.ssla_abi_version() == 2


def test_size_queries_without_gpu():
    from ssla_b200 import _lib

    lib = _lib.load()
    assert lib.ssla_chunk_gla_max_chunks(8, 16384) == (16384 + 63 * 8) // 64
    # bf16, K = V = 64: fp32 increments and adjoints plus the 16-bit adjoint copy
    assert lib.ssla_chunk_gla_workspace_bytes(8, 16384, 4, 64, 64, 1, 1) >= 263 * 4 * 64 * 64 * (4 + 4 + 2)
    # the states buffer holds fp32 and 16-bit chunk-start states on the tensor-core path only
    tc = lib.ssla_chunk_gla_states_bytes(8, 16384, 4, 64, 64, 1, 1)
    simt = lib.ssla_chunk_gla_states_bytes(8, 16384, 4, 64, 64, 0, 0)
    assert simt >= 263 * 4 * 64 * 64 * 4 and tc - simt >= 263 * 4 * 64 * 64 * 2


def test_invalid_args_report_errors():
    from ssla_b200 import _lib

    lib = _lib.load()
    rc = lib.ssla_scan_fwd(None, 7, None, 0, None, 0, None, 1, 1, 1, None)
    assert rc == -1
    assert b"dtype" in lib.ssla_last_error()
    rc = lib.ssla_chunk_gla_fwd(None, None, None, None, 0, 0, None, 1, 10, 1, 300, 300, 1.0,
                                None, None, None, None, 0, None, 0, None)
    assert rc == -1 and b"not supported" in lib.ssla_last_error()


def test_chunk_gla_initial_state_count_valueerror():
    from ssla_b200.ops.gla.chunk import chunk_gla

    q = torch.zeros(8, 1, 4)
    with pytest.raises(ValueError, match="number of initial states"):
        chunk_gla(q, q, q, q, torch.tensor([0, 4, 8]), initial_state=torch.zeros(3, 1, 4, 4))


def test_cpu_tensors_are_rejected():
    from ssla_b200.ops.common.scan import scan

    with pytest.raises(RuntimeError, match="CUDA"):
        scan(torch.zeros(4, 2), torch.zeros(4, 2), torch.tensor([0, 4]))
