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


def test_argument_validation_of_fused_entries():
    """The radial-basis GEMMs and the node-map kernels reject bad arguments on the host, before any
    device work (the device pointers below are never dereferenced)."""
    import numpy as np

    lib = _lib.load()
    dev = ctypes.c_void_p(4096)   # stands in for a device address
    f = ctypes.c_float
    # C = rbf(d) B^T: empty is a no-op, negative sizes / missing operands are invalid
    assert lib.e2a_gemm_tf32x3_rbf(dev, dev, f(-1.0), dev, None, 256, dev, 128, None, 0, 128, 256, 3, None) == 0
    assert lib.e2a_gemm_tf32x3_rbf(dev, dev, f(-1.0), dev, None, 256, dev, 128, None, -5, 128, 256, 3, None) == 1
    assert lib.e2a_gemm_tf32x3_rbf(None, dev, f(-1.0), dev, None, 256, dev, 128, None, 10, 128, 256, 3, None) == 1
    assert lib.e2a_gemm_tf32x3_rbf(dev, dev, f(-1.0), dev, None, 256, dev, 128, None, 10, 128, 256, 2, None) == 1
    # the distance gradient needs ceil(N / 64) partial columns per row
    assert lib.e2a_gemm_tf32x3_rbf_dist_grad(dev, 128, dev, None, 128, dev, dev, f(-1.0), dev, 3, 10, 256, 128, 3,
                                             None) == 1
    j1, j2 = np.eye(3), np.eye(5)
    sel = np.zeros(20, dtype=np.int32)
    cg = np.ones(20)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    assert lib.e2a_node_map_fwd(dev, -1, P(j1), P(j2), P(sel), P(cg), None, dev, None) == 1
    assert lib.e2a_node_map_fwd(dev, 0, None, None, None, None, None, dev, None) == 0
    assert lib.e2a_node_map_fwd(dev, 4, None, P(j2), P(sel), P(cg), None, dev, None) == 1
    bad_sel = sel.copy()
    bad_sel[3] = 9
    assert lib.e2a_node_map_fwd(dev, 4, P(j1), P(j2), P(bad_sel), P(cg), None, dev, None) == 1
    dup = np.arange(20, dtype=np.int32)
    dup[5] = 4
    assert lib.e2a_node_map_fwd(dev, 4, P(j1), P(j2), P(sel), P(cg), P(dup), dev, None) == 1
    assert lib.e2a_node_map_bwd(dev, dev, 4, P(j1), P(j2), P(sel), P(cg), P(dup), dev, None) == 1


def test_ops_refuse_cpu_tensors():
    import pytest
    import torch

    from ubio_molfm_b200 import ops

    with pytest.raises(ValueError):
        ops.prepare_sparse_qk_edge_index_metadata(torch.zeros(3, dtype=torch.long), torch.zeros(3, dtype=torch.long),
                                                  3, 3)
