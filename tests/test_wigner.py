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

def test_fused_output_weights_cache_follows_the_parameters():
    """The merged output-linear weights of the inference path are formed once and re-formed whenever a
    source tensor changes: in place, through load_state_dict, or by a dtype conversion."""
    from ubio_molfm_b200.attention import E2AttentionArbOrder_sparse

    layer = E2AttentionArbOrder_sparse("32x0e+32x1e+32x2e", 32, num_attn_heads=8, attn_scalar_head=8,
                                       irreps_head="4x0e+4x1e+4x2e", alpha_drop=0.0, tp_type="QK_alpha",
                                       attn_type="so2-first-order").eval()
    w1 = layer._fused_out_weights()
    assert all(a is b for a, b in zip(w1, layer._fused_out_weights()))
    with torch.no_grad():
        layer.proj_first.weight.mul_(2.0)
    w2 = layer._fused_out_weights()
    assert all(torch.allclose(b, 2 * a) for a, b in zip(w1, w2))
    sd = {k: v.clone() for k, v in layer.state_dict().items()}
    sd["proj_first.weight"].mul_(0.5)
    layer.load_state_dict(sd)
    assert all(torch.allclose(b, a) for a, b in zip(w1, layer._fused_out_weights()))
    layer.to(torch.float64)
    assert layer._fused_out_weights()[0].dtype == torch.float64
