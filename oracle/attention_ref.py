"""CPU oracle for the E2Former-V2 attention path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
module, and only as the checker / CPU baseline; the product (``ubio_molfm_b200``) never does.

It restates, in plain PyTorch on the CPU, the reference's pure-PyTorch attention path
(``tp_type="QK_alpha"`` without Triton) from IQuestLab/UBio-MolFM, citing the lines it follows
(e2f = src/molfm/models/e2former):

* kernel-level torch fallbacks: ``_torch_sparse_qk_edge_index`` (e2f/e2former.py:63-66),
  ``_torch_sparse_v_agg_edge_index`` / ``edge_agg_kernel`` (e2f/e2former.py:69-77, 393-407),
  the segment sum (e2f/e2former.py:357-363) and the edge-degree outer product
  (e2f/e2former.py:742-749);
* the segmented softmax span (e2f/e2former.py:311-364, 422);
* the full layer forward (e2f/e2former.py:223-436) with ``SO3_Linear_e2former``
  (e2f/module_utils.py:2010-2055), ``SO3_Linear2Scalar_e2former`` (2198-2274), ``RadialProfile``
  (2151-2178) and ``E2TensorProductSO2_FirstOrder`` (e2f/wigner6j/so2_tensor_product.py:182-389).

Parity of this restatement is pinned against golden vectors produced by running the reference's
own code (``tests/golden/make_golden.py``); gradients come from torch autograd.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


# ---------------------------------------------------------------------------------------------
# Kernel-level ops (torch fallbacks of the reference)
# ---------------------------------------------------------------------------------------------
def sparse_qk(query, key, query_index, neighbor_index):
    """e2f/e2former.py:63-66"""
    return torch.sum(query[query_index.long()] * key[neighbor_index.long()], dim=-1)


def v_agg(value, alpha, query_index, value_index, num_queries):
    """e2f/e2former.py:398-407 (scatter_add over the destination)."""
    w = value[value_index.long()] * alpha.unsqueeze(1)
    out = torch.zeros((num_queries, w.shape[1], w.shape[2]), dtype=w.dtype)
    out.scatter_add_(0, query_index.long().view(-1, 1, 1).expand_as(w), w)
    return out


def alpha_sum(alpha, query_index, num_queries):
    """e2f/e2former.py:357-363"""
    out = torch.zeros((num_queries, alpha.shape[1]), dtype=alpha.dtype)
    out.scatter_add_(0, query_index.long().unsqueeze(-1).expand(-1, alpha.shape[1]), alpha)
    return out


def edge_outer(edge_sh, edge_fea, query_index, num_queries):
    """e2f/e2former.py:742-749"""
    outer = edge_sh.unsqueeze(-1) * edge_fea.unsqueeze(1)
    out = torch.zeros((num_queries, edge_sh.shape[1], edge_fea.shape[-1]), dtype=outer.dtype)
    out.index_add_(0, query_index.long(), outer)
    return out


def attention_span(q_scaled, key, value, edge_gate, poly, dist, query_idx, neighbor_idx, num_queries):
    """QK -> gated segmented softmax -> alpha/r -> value aggregation (e2f/e2former.py:311-364, 422,
    so2_tensor_product.py:370-377).  ``value`` is [M, C, H]; ``edge_gate`` [E, 2H]."""
    H = q_scaled.shape[1]
    gate, inputhead = edge_gate[:, :H], edge_gate[:, H:]
    qi = query_idx.long()
    alpha = gate * sparse_qk(q_scaled, key, query_idx, neighbor_idx)
    idx = qi.unsqueeze(-1).expand(-1, H)
    amax = torch.full((num_queries, H), -torch.inf, dtype=alpha.dtype)
    amax = amax.scatter_reduce(0, idx, alpha, reduce="amax", include_self=True)
    alpha = torch.exp(alpha - amax[qi]) * poly.unsqueeze(-1)
    asum = torch.zeros((num_queries, H), dtype=alpha.dtype).scatter_add(0, idx, alpha)
    alpha = alpha * inputhead / (asum[qi] + 1e-3)
    alpha = alpha / dist.unsqueeze(-1).clamp_min(1e-6)
    return v_agg(value, alpha, query_idx, neighbor_idx, num_queries)


# ---------------------------------------------------------------------------------------------
# Layer pieces (functional, over a parameter dict with the reference's state_dict keys)
# ---------------------------------------------------------------------------------------------
def _expand_index(lmax):
    return torch.tensor([l for l in range(lmax + 1) for _ in range(2 * l + 1)])


def so3_linear(x, weight, bias):
    """e2f/module_utils.py:2035-2052"""
    w = torch.index_select(weight, 0, _expand_index(weight.shape[0] - 1))
    out = torch.einsum("bmi, moi -> bmo", x, w)
    out = torch.cat([out[:, :1] + bias.view(1, 1, -1), out[:, 1:]], dim=1)
    return out


def _mlp(x, p, prefix, n_linear):
    """Linear -> LayerNorm -> SiLU ... -> Linear with nn.Sequential indices (module_utils.py:2151)."""
    k = 0
    for li in range(n_linear):
        x = F.linear(x, p[f"{prefix}.{k}.weight"], p[f"{prefix}.{k}.bias"])
        if li == n_linear - 1:
            break
        x = F.layer_norm(x, (x.shape[-1],), p[f"{prefix}.{k + 1}.weight"], p[f"{prefix}.{k + 1}.bias"])
        x = F.silu(x)
        k += 3
    return x


def so3_linear2scalar(x, p, prefix):
    """e2f/module_utils.py:2240-2274"""
    lmax = p[f"{prefix}.weight"].shape[0] - 1
    ei = _expand_index(lmax)
    w = torch.index_select(p[f"{prefix}.weight"], 0, ei)
    out = torch.einsum("bmi, moi -> bmo", x, w)
    out = torch.cat([out[:, :1] + p[f"{prefix}.bias"], out[:, 1:]], dim=1)
    w2 = torch.index_select(p[f"{prefix}.weight2"], 0, ei)
    out2 = torch.einsum("bmi, moi -> bmo", x, w2)
    parts = [torch.sum(out[:, l * l:(l + 1) ** 2] * out2[:, l * l:(l + 1) ** 2], dim=1) for l in range(lmax + 1)]
    h = torch.cat(parts, dim=-1)
    h = F.linear(h, p[f"{prefix}.final_linear.0.weight"], p[f"{prefix}.final_linear.0.bias"])
    h = F.layer_norm(h, (h.shape[-1],), p[f"{prefix}.final_linear.1.weight"], p[f"{prefix}.final_linear.1.bias"])
    h = F.silu(h)
    return F.linear(h, p[f"{prefix}.final_linear.3.weight"], p[f"{prefix}.final_linear.3.bias"])


def so2_select(x, p):
    """so2_tensor_product.py:263-267"""
    pre = "first_order_tp.so2_tp"
    return x[:, p[f"{pre}.selected_idx"].long()] * p[f"{pre}.CG_weight"].reshape(1, -1, 1)


def so2_forward_linear(y, p, l3_sequential):
    """so2_tensor_product.py:273-290"""
    pre = "first_order_tp.so2_tp"
    bs = y.shape[0]
    start = 0
    outs = []
    for idx, (l3, cnt) in enumerate(l3_sequential):
        end = start + (2 * l3 + 1) * cnt
        blk = y[:, start:end].reshape(bs, cnt, 2 * l3 + 1, -1).permute(0, 2, 1, 3).reshape(bs, 2 * l3 + 1, -1)
        outs.append(F.linear(blk, p[f"{pre}.out_linear.{idx}.weight"]))
        start = end
    return torch.cat(outs, dim=1) * p[f"{pre}.path_norm"]


L3_SEQUENTIAL = [[0, 1], [1, 3], [2, 2]]


def attention_layer(p, H, D, node_pos, x, edge_dis, attn_weight, atomic_numbers, poly_dist, bd):
    """E2AttentionArbOrder_sparse.forward, QK_alpha / so2-first-order (e2f/e2former.py:223-436)."""
    N1 = x.shape[0]
    outcell = bd["f_outcell_index"].long()
    N2 = outcell.shape[0]
    qi = bd["query_idx"].long()
    ni = bd["neighbor_idx"].long()
    tgt = p["target_embedding.weight"][atomic_numbers.long()]
    src = p["source_embedding.weight"][atomic_numbers.long()][outcell]
    query = so3_linear2scalar(x, p, "query_linear").reshape(N1, H, -1)
    key = so3_linear2scalar(x, p, "key_linear")[outcell].reshape(N2, H, -1)
    x_edge = torch.cat([attn_weight, tgt[qi], src[ni]], dim=-1)
    edge_gate = _mlp(x_edge, p, "fc_easy.net", 3)
    q_scaled = query / math.sqrt(query.shape[-1])
    value = so3_linear(x, p["proj_value.weight"], p["proj_value.bias"])[outcell]
    C = value.shape[-1]
    hb = torch.bmm(bd["wigner_exp"], value)
    hb = so2_select(hb, p) * torch.norm(bd["f_exp_node_pos"], dim=-1).reshape(-1, 1, 1)
    hb = torch.bmm(bd["wigner_inv_exp"], hb)
    nb_ = hb.shape[1]
    merged = torch.cat([hb, value], dim=1).reshape(N2, -1, H)
    agg = attention_span(q_scaled, key, merged, edge_gate, poly_dist, edge_dis, qi, ni, N1).reshape(N1, -1, C)
    hb_agg, ha = agg[:, :nb_], agg[:, nb_:]
    ha = torch.bmm(bd["wigner"], ha)
    ha = so2_select(ha, p) * torch.norm(node_pos, dim=-1).reshape(-1, 1, 1)
    ha = torch.bmm(bd["wigner_inv"], ha)
    out = so2_forward_linear(ha - hb_agg, p, L3_SEQUENTIAL)
    return so3_linear(out, p["proj_first.weight"], p["proj_first.bias"])
