"""Loading helpers for the golden fixtures (test infrastructure)."""
import json
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    return {k: z[k] for k in z.files}


def layer_cfg(rec):
    return json.loads(str(rec["cfg"]))


def build_product_layer(cfg, device="cpu"):
    from ubio_molfm_b200.attention import E2AttentionArbOrder_sparse
    from ubio_molfm_b200.synthetic import seeded_params_

    C = cfg["C"]
    layer = E2AttentionArbOrder_sparse(f"{C}x0e+{C}x1e+{C}x2e", cfg["nb"], num_attn_heads=cfg["H"],
                                       attn_scalar_head=cfg["D"], irreps_head=cfg["head_irreps"], alpha_drop=0.0,
                                       tp_type="QK_alpha", attn_type="so2-first-order")
    seeded_params_(layer, cfg["seed"])
    return layer.to(device).eval()


LEAVES = ["node_pos", "node_irreps_input", "edge_dis", "poly_dist", "f_exp_node_pos", "wigner", "wigner_inv",
          "wigner_exp", "wigner_inv_exp", "attn_weight"]


def layer_inputs(rec, device="cpu", requires_grad=True):
    leaves = {k: torch.tensor(rec[f"in_{k}"], device=device, requires_grad=requires_grad) for k in LEAVES}
    bd = {
        "query_idx": torch.tensor(rec["query_idx"], device=device),
        "neighbor_idx": torch.tensor(rec["neighbor_idx"], device=device),
        "metadata": tuple(torch.tensor(rec[f"md{i}"], device=device) for i in range(6)),
        "f_outcell_index": torch.tensor(rec["f_outcell_index"], device=device),
        "f_exp_node_pos": leaves["f_exp_node_pos"],
        "wigner": leaves["wigner"], "wigner_inv": leaves["wigner_inv"],
        "wigner_exp": leaves["wigner_exp"], "wigner_inv_exp": leaves["wigner_inv_exp"],
    }
    Z = torch.tensor(rec["Z"], device=device)
    return leaves, bd, Z
