"""The CPU oracle against golden vectors produced by the reference's own code (CPU, no GPU)."""
import json
import os

import numpy as np
import pytest
import torch

from golden_io import GOLDEN, LEAVES, build_product_layer, layer_cfg, layer_inputs, load
from oracle import attention_ref as R

LAYER_CASES = ["layer_small_pbc", "layer_full_mol24"]


@pytest.mark.parametrize("name", LAYER_CASES)
def test_oracle_layer_matches_reference(name):
    rec = load(name)
    cfg = layer_cfg(rec)
    p = {k: v.detach() for k, v in build_product_layer(cfg).state_dict().items()}
    leaves, bd, Z = layer_inputs(rec)
    out = R.attention_layer(p, cfg["H"], cfg["D"], leaves["node_pos"], leaves["node_irreps_input"],
                            leaves["edge_dis"], leaves["attn_weight"], Z, leaves["poly_dist"], bd)
    ref = torch.tensor(rec["out"])
    scale = ref.abs().max().item()
    assert (out - ref).abs().max().item() <= 1e-5 * max(scale, 1.0)
    grads = torch.autograd.grad(out, [leaves[k] for k in LEAVES], torch.tensor(rec["dout"]), allow_unused=True)
    for k, g in zip(LEAVES, grads):
        gref = torch.tensor(rec[f"grad_{k}"])
        g = torch.zeros_like(gref) if g is None else g
        tol = 1e-5 * max(gref.abs().max().item(), 1.0)
        assert (g - gref).abs().max().item() <= tol, k


def test_cg_tables_match_reference():
    from ubio_molfm_b200.cg import so2_first_order_tables

    pin = json.load(open(os.path.join(GOLDEN, "so2_pin.json")))
    assert pin["max_abs_diff"] < 1e-5  # the reference's own node-decomposition identity held
    _, seq, sel, w, _ = so2_first_order_tables()
    assert seq == pin["l3_sequential"]
    assert sel == pin["selected_idx"]
    np.testing.assert_allclose(w, pin["CG_weight"], atol=1e-7)
