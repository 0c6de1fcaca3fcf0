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


def _oracle_graph(rec, cfg):
    """The graph of a backbone fixture from the C graph oracle (pinned bit-exact to the reference)."""
    from oracle import graph_ref
    from ubio_molfm_b200.graph import pbc_image_offsets

    pos = rec["pos"].astype(np.float32)
    n = len(pos)
    pbc = [bool(v) for v in rec["pbc"]]
    cutoff, maxnb = cfg["max_radius"], cfg["max_neighbors"]
    if any(pbc):
        off = pbc_image_offsets(rec["cell"], pbc, cutoff).numpy()
        ia = graph_ref.pbc_expand(pos, off, cutoff)
        outcell, offsets = ia % n, off[ia // n]
        exp = (pos[outcell] + offsets).astype(np.float32)
        qi, ni, _ = graph_ref.radius_graph(pos, exp, [0, n], [0, len(exp)], cutoff, 1e-4, maxnb)
        return qi, ni, outcell, offsets, True, None
    counts = np.bincount(rec["batch"])
    ptr = np.concatenate([[0], np.cumsum(counts)])
    qi, ni, _ = graph_ref.radius_graph(pos, pos, ptr, ptr, cutoff, 1e-4, maxnb)
    return qi, ni, np.arange(n), None, False, torch.tensor(rec["batch"])


@pytest.mark.parametrize("name", ["backbone_pbc40", "backbone_mol3"])
def test_model_oracle_matches_reference(name):
    """The CPU restatement of the full energy + forces evaluation against the reference's own model."""
    import json

    from oracle import model_ref as M
    from ubio_molfm_b200.model import E2FormerPotential
    from ubio_molfm_b200.synthetic import seeded_params_

    rec = load(name)
    cfg = json.loads(str(rec["cfg"]))
    seed = cfg.pop("seed")
    cfg.pop("head")
    m = E2FormerPotential(**cfg)          # parameter names / shapes only (CPU, never run)
    seeded_params_(m.decoder, seed)
    seeded_params_(m.energy_head, seed + 1)
    p = {k: v.detach() for k, v in m.decoder.state_dict().items()}
    ph = {k: v.detach() for k, v in m.energy_head.state_dict().items()}
    qi, ni, outcell, offsets, pbc_any, batch = _oracle_graph(rec, cfg)
    graph = (torch.tensor(qi), torch.tensor(ni), torch.tensor(outcell),
             None if offsets is None else torch.tensor(offsets), pbc_any)
    energy, forces, x = M.energy_forces(p, ph, cfg, torch.tensor(rec["pos"]), torch.tensor(rec["Z"]), graph, batch)
    n_atoms = torch.tensor(np.bincount(rec["batch"]), dtype=torch.float64)
    e_ref = torch.tensor(rec["energy"], dtype=torch.float64)
    assert bool((((energy.double() - e_ref) / n_atoms).abs() <= 1e-6 * (e_ref / n_atoms).abs() + 1e-7).all())
    assert (forces.double() - torch.tensor(rec["forces"], dtype=torch.float64)).abs().max().item() <= 1e-5
    xr = torch.tensor(rec["node_irreps"])
    assert (x - xr).abs().max().item() <= 1e-5 * max(1.0, xr.abs().max().item())
