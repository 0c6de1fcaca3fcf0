"""Host-side logic of the inference path that needs no GPU."""
import pytest
import torch


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


def test_create_graph_needs_training_mode():
    """Force-loss training (forces with their graph) runs in training mode; the eval-mode fused ops are
    first-order only, so asking for a graph in eval mode is refused before any device work."""
    import torch

    from ubio_molfm_b200.model import E2FormerPotential

    m = E2FormerPotential(irreps_node_embedding="32x0e+32x1e+32x2e", num_layers=1, number_of_basis=32,
                          num_attn_heads=8, attn_scalar_head=8, irreps_head="4x0e+4x1e+4x2e", alpha_drop=0.0).eval()
    with pytest.raises(RuntimeError, match="training mode"):
        m(torch.zeros(3, 3), torch.ones(3, dtype=torch.long), create_graph=True)
