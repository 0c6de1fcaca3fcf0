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


def _system_model(rec):
    from ubio_molfm_b200.model import E2FormerPotential
    from ubio_molfm_b200.synthetic import SYSTEM_EMBED_GAINS, seeded_params_

    cfg = json.loads(str(rec["cfg"]))
    seed = cfg.pop("seed")
    cfg.pop("head")
    m = E2FormerPotential(**cfg)
    seeded_params_(m.backbone, seed, gains=SYSTEM_EMBED_GAINS)   # names as in the reference backbone
    seeded_params_(m.energy_head, seed + 1)
    return m, cfg


@pytest.mark.parametrize("name", ["system_pbc40", "system_mol4"])
def test_model_oracle_with_charge_matches_reference_backbone(name):
    """The CPU restatement, charge / multiplicity embedding included, against the reference's own
    ``E2FormerBackbone`` (e2former_wrapper.py:140-339) + energy head on the collated input layout."""
    from oracle import model_ref as M

    rec = load(name)
    m, cfg = _system_model(rec)
    p = {k: v.detach() for k, v in m.decoder.state_dict().items()}
    ps = {k: v.detach() for k, v in m.backbone.state_dict().items() if not k.startswith("decoder.")}
    ph = {k: v.detach() for k, v in m.energy_head.state_dict().items()}
    qi, ni, outcell, offsets, pbc_any, batch = _oracle_graph(rec, cfg)
    graph = (torch.tensor(qi), torch.tensor(ni), torch.tensor(outcell),
             None if offsets is None else torch.tensor(offsets), pbc_any)
    args = (p, ph, cfg, torch.tensor(rec["pos"]), torch.tensor(rec["Z"]), graph, batch)
    energy, forces, x = M.energy_forces(*args, p_system=ps, charge=rec["charge"], multiplicity=rec["multiplicity"])
    n_atoms = torch.tensor(np.bincount(rec["batch"]), dtype=torch.float64)
    e_ref = torch.tensor(rec["energy"], dtype=torch.float64)
    assert bool((((energy.double() - e_ref) / n_atoms).abs() <= 1e-6 * (e_ref / n_atoms).abs() + 1e-7).all())
    assert (forces.double() - torch.tensor(rec["forces"], dtype=torch.float64)).abs().max().item() <= 1e-5
    xr = torch.tensor(rec["node_irreps"])
    assert (x - xr).abs().max().item() <= 1e-5 * max(1.0, xr.abs().max().item())
    # the system embedding is not a no-op on these fixtures: without it the energies move
    e0, _, _ = M.energy_forces(*args)
    assert ((e0.double() - e_ref).abs() / n_atoms).min().item() > 1e-4
    _, f0, _ = M.energy_forces(*args)
    assert (f0.double() - torch.tensor(rec["forces"], dtype=torch.float64)).abs().max().item() > 1e-3


@pytest.mark.parametrize("name", ["system_pbc40", "system_mol4"])
def test_backbone_state_dict_layout_matches_reference(name):
    """Every key and shape of the reference ``E2FormerBackbone`` state dict, recorded by the generator,
    exists here (but the constants the model does not read); a strict load of a state dict with exactly that layout works, as does the
    ``MolfmAtomic`` layout (``decoder.*`` + ``head.energy_heads.<name>.mlp.*``)."""
    rec = load(name)
    m, _ = _system_model(rec)
    ref = json.loads(str(rec["state_dict_shapes"]))
    mine = {k: list(v.shape) for k, v in m.backbone.state_dict().items()}
    extra = sorted(set(ref) - set(mine))
    # the reference also stores J matrices above lmax and an unused harmonics table: dropped on load
    assert all(k.startswith("decoder.Jd_list.") or k == "decoder.edge_deg_embed_dense.sph.W" for k in extra), extra
    assert {k: v for k, v in ref.items() if k not in extra} == mine
    sd = {k: torch.full(v, 0.25) for k, v in ((k, tuple(s)) for k, s in ref.items())}
    m.backbone.load_state_dict(sd, strict=True)
    assert float(m.backbone.embedding_charge.weight[3, 2]) == 0.25
    full = {"decoder." + k: v for k, v in sd.items()}
    full.update({f"head.energy_heads.omol.{k}": torch.full(v.shape, 1.25) for k, v in m.energy_head.state_dict().items()})
    m.load_reference_state_dict(full)
    assert float(m.energy_head.mlp[0].bias[0]) == 1.25
    with pytest.raises(KeyError):
        m.load_reference_state_dict(full, head_name="spice")
