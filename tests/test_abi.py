"""The C-ABI library loads and exports every entry point declared in include/e2a.h (no GPU needed)."""
import ctypes
import os
import re

from ubio_molfm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "e2a.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(e2a_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_host_only_entry_points():
    lib = _lib.load()
    assert lib.e2a_version() >= 100
    assert lib.e2a_status_string(0) == b"ok"
    assert lib.e2a_status_string(3) == b"workspace too small"
    assert lib.e2a_csr_workspace_bytes(1000, 10, 10) > 0
    assert lib.e2a_attn_bwd_workspace_bytes(1000, 128) >= 2 * 1000 * 128 * 4
    # argument validation happens before any device work
    assert lib.e2a_attn_fwd(None, None, None, None, None, 8, None, None, None, None, None, 4, 4, 0, 6, 8, 4,
                            None, None, None, None, None) == 4  # H % 4 != 0 -> unsupported
    assert lib.e2a_attn_fwd(None, None, None, None, None, 8, None, None, None, None, None, 4, 4, 0, 8, 6, 4,
                            None, None, None, None, None) == 4  # D % 4 != 0
    assert lib.e2a_attn_fwd(None, None, None, None, None, 8, None, None, None, None, None, 4, 4, 0, 8, 8, 4,
                            None, None, None, None, None) == 1  # NULL pointers -> invalid argument


def test_ops_refuse_cpu_tensors():
    import pytest
    import torch

    from ubio_molfm_b200 import ops

    with pytest.raises(ValueError):
        ops.prepare_sparse_qk_edge_index_metadata(torch.zeros(3, dtype=torch.long), torch.zeros(3, dtype=torch.long),
                                                  3, 3)
