"""Per-node Wigner matrices against the reference's (as recorded in the golden layer inputs)."""
import numpy as np
import pytest
import torch

from golden_io import load


@pytest.mark.parametrize("name", ["layer_small_pbc", "layer_full_mol24"])
def test_node_wigner_matches_reference(name):
    from ubio_molfm_b200.wigner import node_wigner

    rec = load(name)
    W, Wi = node_wigner(torch.tensor(rec["in_node_pos"]))
    np.testing.assert_allclose(W.numpy(), rec["in_wigner"], atol=1e-6)
    np.testing.assert_allclose(Wi.numpy(), rec["in_wigner_inv"], atol=1e-6)
    We, Wie = node_wigner(torch.tensor(rec["in_f_exp_node_pos"]))
    np.testing.assert_allclose(We.numpy(), rec["in_wigner_exp"], atol=1e-6)
    np.testing.assert_allclose(Wie.numpy(), rec["in_wigner_inv_exp"], atol=1e-6)


def test_wigner_gradient_finite_at_origin_and_pole():
    from ubio_molfm_b200.wigner import node_wigner

    pos = torch.tensor([[0.0, 0.0, 0.0], [0.0, 2.0, 0.0], [0.3, -1.0, 0.7]], dtype=torch.float64,
                       requires_grad=True)
    W, Wi = node_wigner(pos, dtype=torch.float64)
    (g,) = torch.autograd.grad((W ** 2).sum() + Wi.sum(), pos)
    assert torch.isfinite(g).all()


def test_jd_matches_reference_constants():
    """The computed J matrices against the reference's ``Jd.pt`` (fixture written by
    ``tests/golden/make_golden.py jd``)."""
    from golden_io import load
    from ubio_molfm_b200.wigner import jd_matrices

    ref = load("jd_reference")
    for l, J in enumerate(jd_matrices(2)):
        np.testing.assert_allclose(J.numpy(), ref[f"J{l}"], atol=1e-12)
