"""Generate the golden fixtures under ``tests/golden/`` by running the REFERENCE code on CPU.

TEST INFRASTRUCTURE ONLY.  Run in a container where the reference sources are mounted
(``E2A_REFERENCE_ROOT`` = the reference checkout, the directory holding ``src/molfm``)::

    E2A_REFERENCE_ROOT=<reference checkout> python tests/golden/make_golden.py [graph|layer|backbone|faiss|system]

It imports the reference's own modules through ``refshim`` (stand-ins for the missing third-party
packages) and records, as compressed ``.npz`` files:

* ``graph_*.npz`` -- ``CellExpander.expand_includeself`` (module_utils.py:1065-1275) and
  ``construct_radius_neighbor`` (module_utils.py:3119-3242) outputs: expanded positions, image
  -> atom map, edge lists, distances, edge vectors, envelope values and the CSR metadata of
  ``prepare_sparse_qk_edge_index_metadata`` (triton_sparse_qk_autograd.py:635-652).
* ``layer_*.npz`` -- ``E2AttentionArbOrder_sparse.forward`` (e2former.py:223-436) with
  ``tp_type="QK_alpha"`` / ``attn_type="so2-first-order"`` on seeded inputs and seeded weights
  (:func:`ubio_molfm_b200.synthetic.seeded_params_`), plus the gradients of ``<out, dOut>`` with
  respect to every floating-point input, for a seeded ``dOut``.
* ``faiss_expand_*.npz`` -- ``distributed_cell_expand`` (sp/dist_ner.py:27-84), the image expansion of
  the reference's FAISS neighbour path, with the atoms' bounding box as the wrapper passes it
  (e2former_wrapper.py:179-191): expanded positions and the image -> atom map.
* ``jd_reference.npz`` -- the reference's ``Jd.pt`` (the J matrices of its Wigner construction,
  module_utils.py:266-337), degrees 0..2, as stored.
* ``so2_pin.json`` -- the reference's own identity check ``test_so2_o1`` (so2_tensor_product.py:
  392-478), restated with the current ``eulers_to_wigner`` return convention: the node-decomposed
  first-order TP equals the per-edge rotated TP.

Weights are not stored: tests regenerate them with the same seeded function.
"""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import refshim  # noqa: E402
from ubio_molfm_b200 import synthetic  # noqa: E402

torch.set_default_dtype(torch.float32)


def _np(t):
    return t.detach().cpu().numpy()


def reference_graph(mods, pos, Z, cell, pbc, cutoff, max_neighbors, batch_sizes=None):
    """Run the reference PBC expansion + dense radius graph. ``pos`` is [B,L,3] padded."""
    mu = mods["mu"]
    qkmod = mods["qk"]
    pos = torch.as_tensor(pos, dtype=torch.float32)
    B, L = pos.shape[:2]
    Z = torch.as_tensor(Z, dtype=torch.long)
    node_mask = Z != 0
    padding_mask = ~node_mask
    pos = torch.where(padding_mask.unsqueeze(-1).repeat(1, 1, 3), 999.0, pos)
    cell = torch.as_tensor(cell, dtype=torch.float32)
    pbc_t = torch.as_tensor(pbc, dtype=torch.bool)
    if bool(pbc_t.any()):
        ce = mu.CellExpander(cutoff, 512, 4)
        ex = ce.expand_includeself(pos, pbc_t, Z, cell, neighbors_radius=(None, cutoff),
                                   use_grad=False, padding_mask=padding_mask)
    else:
        ex = {"expand_node_pos": pos, "outcell_index": torch.arange(L).unsqueeze(0).repeat(B, 1),
              "expand_node_mask": node_mask}
    exp_pos = ex["expand_node_pos"].masked_fill(~ex["expand_node_mask"].unsqueeze(-1), 999)
    ptr = torch.nn.functional.pad(node_mask.sum(-1).to(torch.int32).cumsum(0), (1, 0))
    f_exp_node_pos = exp_pos[ex["expand_node_mask"]]
    f_outcell_index = (ex["outcell_index"] + ptr[:B, None])[ex["expand_node_mask"]]
    nb = mu.construct_radius_neighbor(pos, node_mask, exp_pos, ex["expand_node_mask"],
                                      max_dist=cutoff, min_dist=1e-4, max_neighbors=max_neighbors)
    md = nb["metadata"]
    return {
        "pos": _np(pos[node_mask]),
        "Z": _np(Z[node_mask]),
        "batch_ptr": _np(ptr),
        "exp_ptr": _np(torch.nn.functional.pad(ex["expand_node_mask"].sum(-1).cumsum(0), (1, 0))),
        "f_exp_node_pos": _np(f_exp_node_pos),
        "f_outcell_index": _np(f_outcell_index),
        "query_idx": _np(nb["query_idx"]).astype(np.int64),
        "neighbor_idx": _np(nb["neighbor_idx"]).astype(np.int64),
        "f_edge_vec": _np(nb["f_edge_vec"]),
        "f_dist": _np(nb["f_dist"]),
        "f_poly_dist": _np(nb["f_poly_dist"]),
        **{f"md{i}": _np(m) for i, m in enumerate(md)},
    }


def pad_systems(systems):
    """List of (pos, Z) -> padded [B,L,3], [B,L] with Z=0 padding."""
    B = len(systems)
    L = max(len(z) for _, z in systems)
    P = np.zeros((B, L, 3), np.float32)
    ZZ = np.zeros((B, L), np.int64)
    for b, (p, z) in enumerate(systems):
        P[b, : len(z)] = p
        ZZ[b, : len(z)] = z
    return P, ZZ


def graph_cases(mods):
    cases = {}
    # 648-atom water box (the CPU plumbing workload), cutoff 5.0, no neighbour cap.
    pos, Z, cell = synthetic.water_box(seed=0)
    cases["graph_water648"] = reference_graph(mods, pos[None], Z[None], cell[None],
                                              [[True, True, True]], 5.0, None)
    # 1,500-atom biomolecular box, cutoff 4.5, max_neighbors 32 (the full-backbone workload).
    pos, Z, cell = synthetic.bio_box(1500, seed=1)
    cases["graph_bio1500"] = reference_graph(mods, pos[None], Z[None], cell[None],
                                             [[True, True, True]], 4.5, 32)
    # Small periodic box where cutoff > half the box (many images per atom, exact ties possible).
    rng = np.random.default_rng(2)
    pos = rng.uniform(0, 7.0, size=(40, 3))
    Z = rng.choice([1, 6, 8], size=40)
    cases["graph_smallpbc40"] = reference_graph(mods, pos[None], Z[None], (np.eye(3) * 7.0)[None],
                                                [[True, True, True]], 5.0, None)
    # Triclinic cell, mixed pbc (periodic in x,y only).
    cellt = np.array([[9.0, 0.0, 0.0], [2.5, 8.0, 0.0], [1.0, 1.5, 10.0]])
    frac = rng.uniform(0, 1, size=(60, 3))
    pos = frac @ cellt
    Z = rng.choice([1, 6, 7, 8], size=60)
    cases["graph_triclinic60"] = reference_graph(mods, pos[None], Z[None], cellt[None],
                                                 [[True, True, False]], 5.0, 24)
    # Batch of three non-periodic molecules with a neighbour cap (top-K truncation).
    mols = synthetic.molecule_batch(3, 10, 30, seed=3)
    P, ZZ = pad_systems([(m[0], m[1]) for m in mols])
    cases["graph_mol3"] = reference_graph(mods, P, ZZ, np.zeros((3, 3, 3)), [[False] * 3] * 3, 4.0, 8)
    # Lattice with exact distance ties (simple cubic, spacing 2.0, cutoff 4.1, cap 10).
    g = np.arange(4) * 2.0
    pos = np.stack(np.meshgrid(g, g, g, indexing="ij"), -1).reshape(-1, 3)
    Z = np.full(len(pos), 6)
    cases["graph_lattice64"] = reference_graph(mods, pos[None], Z[None], (np.eye(3) * 8.0)[None],
                                               [[True, True, True]], 4.1, 10)
    return cases


def layer_case(mods, name, C, H, D, head_irreps, nb, cutoff, pos, Z, cell, pbc, max_neighbors, seed):
    mu, e2f = mods["mu"], mods["e2f"]
    g = reference_graph(mods, pos[None], Z[None], cell[None], [pbc], cutoff, max_neighbors)
    irreps = f"{C}x0e+{C}x1e+{C}x2e"
    layer = e2f.E2AttentionArbOrder_sparse(
        irreps, nb, num_attn_heads=H, attn_scalar_head=D, irreps_head=head_irreps,
        alpha_drop=0.0, tp_type="QK_alpha", attn_type="so2-first-order", atom_type_cnt=256)
    layer.eval()
    synthetic.seeded_params_(layer, seed)
    l3_seq = layer.first_order_tp.so2_tp.l3_sequential
    Jd = [j.double() for j in torch.load(os.path.join(refshim.E2F_DIR, "Jd.pt"))]

    pos_t = torch.tensor(g["pos"])
    exp_t = torch.tensor(g["f_exp_node_pos"])
    W, Wi = mu.eulers_to_wigner(mu.init_edge_rot_euler_angles(pos_t.double(), training=False), 0, 2, Jd, l3_seq)
    if any(pbc):
        We, Wie = mu.eulers_to_wigner(mu.init_edge_rot_euler_angles(exp_t.double(), training=False), 0, 2, Jd, l3_seq)
    else:
        We, Wie = W, Wi
    rbf = mu.GaussianSmearing(nb, cutoff=cutoff, basis_width_scalar=2)

    gen = torch.Generator().manual_seed(seed + 17)
    N = pos_t.shape[0]
    x = torch.randn((N, 9, C), generator=gen)
    leaves = {
        "node_pos": pos_t.clone(),
        "node_irreps_input": x,
        "edge_dis": torch.tensor(g["f_dist"]),
        "poly_dist": torch.tensor(g["f_poly_dist"]),
        "f_exp_node_pos": exp_t.clone(),
        "wigner": W.float(), "wigner_inv": Wi.float(),
        "wigner_exp": We.float(), "wigner_inv_exp": Wie.float(),
    }
    leaves["attn_weight"] = rbf(leaves["edge_dis"]).detach()
    for v in leaves.values():
        v.requires_grad_(True)
    qi = torch.tensor(g["query_idx"])
    ni = torch.tensor(g["neighbor_idx"])
    md = tuple(torch.tensor(g[f"md{i}"]) for i in range(6))
    bd = {"query_idx": qi, "neighbor_idx": ni, "metadata": md,
          "f_outcell_index": torch.tensor(g["f_outcell_index"]),
          "f_exp_node_pos": leaves["f_exp_node_pos"],
          "wigner": leaves["wigner"], "wigner_inv": leaves["wigner_inv"],
          "wigner_exp": leaves["wigner_exp"], "wigner_inv_exp": leaves["wigner_inv_exp"]}
    out, _ = layer(node_pos=leaves["node_pos"], node_irreps_input=leaves["node_irreps_input"],
                   edge_dis=leaves["edge_dis"], edge_vec=torch.tensor(g["f_edge_vec"]),
                   attn_weight=leaves["attn_weight"], atomic_numbers=torch.tensor(g["Z"]),
                   poly_dist=leaves["poly_dist"], batched_data=bd)
    dout = torch.randn(out.shape, generator=gen)
    grads = torch.autograd.grad(out, list(leaves.values()), dout, allow_unused=True)
    rec = dict(g)
    rec.update({
        "cfg": np.array(json.dumps(dict(C=C, H=H, D=D, head_irreps=head_irreps, nb=nb, cutoff=cutoff,
                                        seed=seed, pbc=list(pbc), max_neighbors=max_neighbors))),
        "out": _np(out), "dout": _np(dout),
    })
    for (k, v), gr in zip(leaves.items(), grads):
        rec[f"in_{k}"] = _np(v)
        rec[f"grad_{k}"] = np.zeros(v.shape, np.float32) if gr is None else _np(gr)
    return rec


def layer_cases(mods):
    cases = {}
    rng = np.random.default_rng(5)
    pos = rng.uniform(0, 7.5, size=(36, 3))
    Z = rng.choice([1, 6, 7, 8], size=36)
    cases["layer_small_pbc"] = layer_case(mods, "small", 32, 8, 8, "4x0e+4x1e+4x2e", 32, 5.0,
                                          pos, Z, np.eye(3) * 7.5, [True, True, True], None, seed=11)
    mols = synthetic.molecule_batch(1, 24, 24, seed=6)
    cases["layer_full_mol24"] = layer_case(mods, "full", 256, 128, 8, "2x0e+2x1e+2x2e", 256, 6.0,
                                           mols[0][0], mols[0][1], np.zeros((3, 3)), [False] * 3, None,
                                           seed=12)
    return cases


BACKBONE_CFG = dict(irreps_node_embedding="32x0e+32x1e+32x2e", num_layers=2, max_neighbors=None,
                    max_radius=5.0, number_of_basis=32, num_attn_heads=8, attn_scalar_head=8,
                    irreps_head="4x0e+4x1e+4x2e", norm_layer="rms_norm_sh", alpha_drop=0.0,
                    tp_type="QK_alpha", attn_type="so2-first-order", atom_type_cnt=256, avg_degree=23.0)


def _energy_head(embedding_dim):
    """The reference's MLP_energy_head (pipeline/head.py:330-341), imported when its module loads
    under the shim; its three-layer MLP otherwise (same parameter names)."""
    try:
        import importlib
        head = importlib.import_module("molfm.pipeline.head")
        return head.MLP_energy_head(embedding_dim, 2), "reference"
    except Exception:  # noqa: BLE001 -- the head module pulls in optional dependencies
        m = torch.nn.Module()
        m.mlp = torch.nn.Sequential(torch.nn.Linear(embedding_dim, embedding_dim), torch.nn.SiLU(),
                                    torch.nn.Linear(embedding_dim, embedding_dim), torch.nn.SiLU(),
                                    torch.nn.Linear(embedding_dim, 1))
        m.forward = lambda emb, irreps=None: m.mlp(emb)
        return m, "restated"


def backbone_case(mods, P, ZZ, cell, pbc, seed, max_neighbors=None):
    """The reference E2former (e2former.py:756-1145) + energy head, energies and forces = -dE/dpos by
    autograd through its own PBC expansion and radius graph (the wrapper's path, e2former_wrapper.py:
    140-339, and GradientHead, pipeline/head.py:305-328)."""
    mu, e2f = mods["mu"], mods["e2f"]
    cfg = dict(BACKBONE_CFG, max_neighbors=max_neighbors)
    dec = e2f.E2former(**cfg).eval()
    synthetic.seeded_params_(dec, seed)
    C = int(cfg["irreps_node_embedding"].split("x")[0])
    head, head_kind = _energy_head(C)
    synthetic.seeded_params_(head, seed + 1)
    P = torch.tensor(P, dtype=torch.float32)
    Z = torch.tensor(ZZ, dtype=torch.long)
    B, L = Z.shape
    node_mask = Z != 0
    padding_mask = ~node_mask
    pos = P.clone().requires_grad_(True)
    posm = torch.where(padding_mask.unsqueeze(-1).repeat(1, 1, 3), 999.0, pos)
    cell_t = torch.tensor(cell, dtype=torch.float32).reshape(1, 3, 3).repeat(B, 1, 1)
    pbc_t = torch.tensor(pbc, dtype=torch.bool).reshape(1, 3).repeat(B, 1)
    bd = {"pos": posm, "atom_masks": node_mask, "atomic_numbers": Z, "pbc": pbc_t, "cell": cell_t}
    if bool(pbc_t.any()):
        ce = mu.CellExpander(cfg["max_radius"], 512, 4)
        ex = ce.expand_includeself(posm, pbc_t, Z, cell_t, neighbors_radius=(None, cfg["max_radius"]),
                                   use_grad=True, padding_mask=padding_mask)
    else:
        ex = {"expand_node_pos": posm, "outcell_index": torch.arange(L).unsqueeze(0).repeat(B, 1),
              "expand_node_mask": node_mask}
    bd.update(ex)
    exp_pos = bd["expand_node_pos"].masked_fill(~bd["expand_node_mask"].unsqueeze(-1), 999)
    bd["expand_node_pos"] = exp_pos
    ptr = torch.nn.functional.pad(node_mask.sum(-1).to(torch.int32).cumsum(0), (1, 0))
    bd["f_exp_node_pos"] = exp_pos[bd["expand_node_mask"]]
    bd["f_outcell_index"] = (bd["outcell_index"] + ptr[:B, None])[bd["expand_node_mask"]]
    nb = mu.construct_radius_neighbor(posm, node_mask, exp_pos, bd["expand_node_mask"],
                                      max_dist=cfg["max_radius"], min_dist=1e-4, max_neighbors=max_neighbors)
    tok = torch.zeros(B, L, C)
    node_attr, _, node_irreps = dec(bd, tok, None, neighbor_info=nb)
    e_atom = head(node_attr, node_irreps).squeeze(-1).masked_fill(~node_mask, 0.0)
    energy = e_atom.sum(dim=-1)
    (grad,) = torch.autograd.grad(energy.sum(), pos)
    return {
        "cfg": np.array(json.dumps(dict(cfg, seed=seed, head=head_kind))),
        "pos": _np(P[node_mask]), "Z": _np(Z[node_mask]),
        "batch": _np(torch.arange(B).unsqueeze(1).repeat(1, L)[node_mask]),
        "cell": np.asarray(cell, np.float32), "pbc": np.asarray(pbc, bool),
        "energy": _np(energy), "forces": _np(-grad[node_mask]),
        "node_irreps": _np(node_irreps[node_mask]), "n_edges": np.array(int(nb["query_idx"].numel())),
    }


def backbone_cases(mods):
    cases = {}
    rng = np.random.default_rng(8)
    pos = rng.uniform(0, 8.0, size=(40, 3)).astype(np.float32)
    Z = rng.choice([1, 6, 7, 8], size=40)
    cases["backbone_pbc40"] = backbone_case(mods, pos[None], Z[None], np.eye(3, dtype=np.float32) * 8.0,
                                            [True, True, True], seed=31)
    mols = synthetic.molecule_batch(3, 8, 20, seed=9)
    P, ZZ = pad_systems([(m[0], m[1]) for m in mols])
    cases["backbone_mol3"] = backbone_case(mods, P, ZZ, np.zeros((3, 3), np.float32), [False] * 3, seed=32,
                                           max_neighbors=12)
    return cases


def system_case(mods, P, ZZ, cell, pbc, charge, mult, seed, max_neighbors=None):
    """The reference's ``E2FormerBackbone`` (e2former_wrapper.py:140-339) -- PBC expansion, radius
    graph, the charge / multiplicity system embedding (``mix_cm``, e2former_wrapper.py:249-259) added to
    the normed l=0 row of every block (e2former.py:582-583) -- plus ``MLP_energy_head`` summed over the
    atoms (pipeline/head.py:552-580) and forces = -dE/dpos (GradientHead, head.py:305-328), on the
    collated input layout of ``dict_to_model_input`` (interface/data_utils.py:37-80: ``pos [B,L,3]``,
    ``atom_masks``, ``charge [B,1]``, ``multiplicity [B,1]``, ``cell [B,3,3]``, ``pbc [B,3]``).  All
    weights of the backbone are seeded by their names in the backbone (``decoder.blocks...``)."""
    import importlib

    wrapper = importlib.import_module("molfm.models.e2former.e2former_wrapper")
    cfg = dict(BACKBONE_CFG, max_neighbors=max_neighbors, encoder="default")
    bb = wrapper.E2FormerBackbone(use_faiss=False, **cfg).eval()
    synthetic.seeded_params_(bb, seed, gains=synthetic.SYSTEM_EMBED_GAINS)
    C = int(cfg["irreps_node_embedding"].split("x")[0])
    head, head_kind = _energy_head(C)
    synthetic.seeded_params_(head, seed + 1)
    P = torch.tensor(P, dtype=torch.float32)
    Z = torch.tensor(ZZ, dtype=torch.long)
    B, L = Z.shape
    node_mask = Z != 0
    pos = P.clone().requires_grad_(True)
    bd = {"pos": pos, "atom_masks": node_mask, "atomic_numbers": Z,
          "pbc": torch.tensor(pbc, dtype=torch.int32).reshape(1, 3).repeat(B, 1),
          "cell": torch.tensor(cell, dtype=torch.float32).reshape(1, 3, 3).repeat(B, 1, 1),
          "charge": torch.tensor(charge, dtype=torch.int32).reshape(B, 1),
          "multiplicity": torch.tensor(mult, dtype=torch.int32).reshape(B, 1)}
    out = bb(bd)
    e_atom = head(out["node_featuresBxN"], out["node_irrepsBxN"]).squeeze(-1).masked_fill(~node_mask, 0.0)
    energy = e_atom.sum(dim=-1)
    (grad,) = torch.autograd.grad(energy.sum(), pos)
    return {
        "cfg": np.array(json.dumps(dict(cfg, seed=seed, head=head_kind))),
        "pos": _np(P[node_mask]), "Z": _np(Z[node_mask]),
        "batch": _np(torch.arange(B).unsqueeze(1).repeat(1, L)[node_mask]),
        "cell": np.asarray(cell, np.float32), "pbc": np.asarray(pbc, bool),
        "charge": np.asarray(charge, np.int64), "multiplicity": np.asarray(mult, np.int64),
        "energy": _np(energy), "forces": _np(-grad[node_mask]),
        "node_irreps": _np(out["node_irrepsBxN"][node_mask]),
        "n_edges": np.array(int(out["neighbor_info"]["query_idx"].numel())),
        "state_dict_shapes": np.array(json.dumps({k: list(v.shape) for k, v in bb.state_dict().items()})),
    }


def system_cases(mods):
    cases = {}
    rng = np.random.default_rng(8)
    pos = rng.uniform(0, 8.0, size=(40, 3)).astype(np.float32)
    Z = rng.choice([1, 6, 7, 8], size=40)
    cases["system_pbc40"] = system_case(mods, pos[None], Z[None], np.eye(3, dtype=np.float32) * 8.0,
                                        [True, True, True], [1], [2], seed=41)
    mols = synthetic.molecule_batch(4, 8, 20, seed=10)
    P, ZZ = pad_systems([(m[0], m[1]) for m in mols])
    cases["system_mol4"] = system_case(mods, P, ZZ, np.zeros((3, 3), np.float32), [False] * 3,
                                       [-1, 0, 1, 0], [1, 2, 1, 1], seed=42, max_neighbors=12)
    return cases


def so2_pin(mods):
    mu, so2tp = mods["mu"], mods["so2tp"]
    torch.manual_seed(0)
    C = 16
    tp = so2tp.SO2_TP_givenl2(l1_list=range(3), l2=1, l3_legal=range(3), in_c=C, out_c=C,
                              with_linear=True).double()
    Jd = [j.double() for j in torch.load(os.path.join(refshim.E2F_DIR, "Jd.pt"))]
    N = 10
    pos = torch.randn(N, 3, dtype=torch.float64)
    h = torch.randn(N, 9, C, dtype=torch.float64)
    alpha = torch.randn(N, N, C, dtype=torch.float64)
    eye = torch.eye(N).bool()
    alpha[eye] = 0
    r = torch.norm(pos[:, None] - pos[None], dim=-1, keepdim=True)
    r[eye] = 1
    adr = alpha / r
    W, Wi = mu.eulers_to_wigner(mu.init_edge_rot_euler_angles(pos, training=False), 0, 2, Jd, tp.l3_sequential)
    nrm = pos.norm(dim=-1).reshape(-1, 1, 1)
    hb = torch.bmm(Wi, tp(torch.bmm(W, h), with_linear=False) * nrm)
    hb = (hb[None] * adr.reshape(N, N, 1, C)).sum(1)
    ha = (h[None] * adr.reshape(N, N, 1, C)).sum(1)
    ha = torch.bmm(Wi, tp(torch.bmm(W, ha), with_linear=False) * nrm)
    out1 = tp.forward_linear(ha - hb)
    ev = pos[:, None] - pos[None]
    ev[eye] = torch.tensor([0.0, 1e-3, 0.0], dtype=torch.float64)
    ev = (ev / ev.norm(dim=-1, keepdim=True)).reshape(-1, 3)
    We, Wie = mu.eulers_to_wigner(mu.init_edge_rot_euler_angles(ev, training=False), 0, 2, Jd, tp.l3_sequential)
    hij = h[None].repeat(N, 1, 1, 1).reshape(N * N, 9, C)
    hij = torch.bmm(Wie, tp(torch.bmm(We, hij), with_linear=False)).reshape(N, N, -1, C)
    out2 = tp.forward_linear((hij * alpha.reshape(N, N, 1, C)).sum(1))
    return {
        "max_abs_diff": float((out1 - out2).abs().max()),
        "selected_idx": tp.selected_idx.tolist(),
        "CG_weight": [float(v) for v in tp.CG_weight.double()],
        "l3_sequential": [list(x) for x in tp.l3_sequential],
    }


def faiss_cases(mods):
    """The FAISS path's image expansion on three periodic systems (CPU, fp32)."""
    import importlib

    dn = importlib.import_module("molfm.models.e2former.sp.dist_ner")
    rng = np.random.default_rng(31)
    systems = {}
    pos, _, cell = synthetic.water_box(n_side=6, box=18.64, jitter=0.3, seed=1)
    systems["faiss_expand_water648"] = (pos, cell, [True, True, True], 5.0)
    tri = np.array([[8.0, 0.0, 0.0], [2.0, 7.0, 0.0], [1.0, 1.5, 9.0]])
    systems["faiss_expand_triclinic60"] = (rng.random((60, 3)) @ tri, tri, [True, True, False], 4.5)
    systems["faiss_expand_small40"] = (rng.random((40, 3)) * 7.0, np.eye(3) * 7.0, [True, True, True], 5.0)
    out = {}
    for name, (p, c, pbc, cutoff) in systems.items():
        pt = torch.tensor(p, dtype=torch.float32).unsqueeze(0)
        ct = torch.tensor(c, dtype=torch.float32)
        bmin, bmax = pt[0].min(dim=0)[0], pt[0].max(dim=0)[0]
        r = dn.distributed_cell_expand(pt, ct, cutoff, bmin, bmax, 1, torch.tensor([pbc]))
        out[name] = {"pos": pt[0].numpy(), "cell": ct.numpy(), "pbc": np.array(pbc), "cutoff": np.array(cutoff),
                     "expand_node_pos": r["expand_node_pos"][0].numpy(),
                     "outcell_index": r["outcell_index"][0].numpy(), "n_edges": np.array(0)}
    return out


def main(only=None):
    """Write every fixture, or only those whose name starts with ``only``."""
    if only in (None, "jd"):
        jd = torch.load(os.path.join(refshim.REF_ROOT, "src", "molfm", "models", "e2former", "Jd.pt"))
        np.savez_compressed(os.path.join(HERE, "jd_reference.npz"),
                            **{f"J{l}": jd[l].double().numpy() for l in range(3)})
        print("jd_reference", [tuple(jd[l].shape) for l in range(3)])
        if only == "jd":
            return
    mods = refshim.load_reference()
    if only is None:
        pin = so2_pin(mods)
        assert pin["max_abs_diff"] < 1e-5, pin
        with open(os.path.join(HERE, "so2_pin.json"), "w") as f:
            json.dump(pin, f, indent=1)
        print("so2 pin", pin["max_abs_diff"])
    makers = {"graph": graph_cases, "layer": layer_cases, "backbone": backbone_cases, "faiss": faiss_cases,
              "system": system_cases}
    for prefix, make in makers.items():
        if only is not None and prefix != only:
            continue
        for name, rec in make(mods).items():
            np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **rec)
            print(name, "N=", len(rec["pos"]), "E=", len(rec["query_idx"]) if "query_idx" in rec else int(rec["n_edges"]))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else None)
