"""CPU oracle for the full E2Former-V2 energy + forces evaluation -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this
module, and only as the checker / CPU baseline; the product (``ubio_molfm_b200``) never does.

A plain-PyTorch CPU restatement, on a flat parameter dict (the backbone's ``state_dict``), of
(e2f = src/molfm/models/e2former, mu = e2f/module_utils.py):

* ``EquivariantRMSNormArraySphericalHarmonicsV2_BL.forward`` (mu:1720-1772);
* ``Gate_s3`` / ``FeedForwardNetwork_s3`` (mu:2694-2797) with e3nn's second-moment normalised SiLU
  and sigmoid (the normalising constants by Gauss-Hermite quadrature of E[f(z)^2], z ~ N(0,1));
* ``EdgeDegreeEmbeddingNetwork_higherorder.forward`` (e2f/e2former.py:689-753, ``use_atom_edge``)
  with e3nn's component-normalised real spherical harmonics for l <= 2 (y the polar axis);
* ``TransBlock.forward`` (e2f/e2former.py:526-620) around :func:`attention_ref.attention_layer`;
* ``E2former.forward`` (e2f/e2former.py:944-1145): per-node Wigner matrices from the Euler angles of
  the absolute positions (mu:182-337), RBF, edge-degree embedding, the blocks, the final norm;
* ``MLP_energy_head`` (pipeline/head.py:330-341) summed over atoms, forces = -dE/dpos
  (pipeline/head.py:305-328) by autograd through the edge geometry.

The J matrices of the Wigner construction are taken from the parameter dict (``Jd_list.*``, the
reference's ``Jd.pt``).  Pinned against the reference's own model through ``tests/golden/backbone_*``.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from . import attention_ref as R


def _sub(p, prefix):
    n = len(prefix)
    return {k[n:]: v for k, v in p.items() if k.startswith(prefix)}


def rms_norm(p, pre, x, lmax, eps=1e-5):
    """mu:1720-1772 (component normalisation, balanced degrees, centred, affine)."""
    f0 = x[:, :1] - x[:, :1].mean(dim=2, keepdim=True)
    f = torch.cat([f0, x[:, 1:]], dim=1)
    bw = torch.tensor([1.0 / (2 * l + 1) / (lmax + 1) for l in range(lmax + 1) for _ in range(2 * l + 1)],
                      dtype=x.dtype).reshape(1, -1, 1)
    norm = torch.mean((f.pow(2) * bw).sum(dim=1, keepdim=True), dim=2, keepdim=True)
    norm = (norm + eps).pow(-0.5)
    w = p[f"{pre}affine_weight"][R._expand_index(lmax)].unsqueeze(0)
    out = f * (norm * w)
    return torch.cat([out[:, :1] + p[f"{pre}affine_bias"].reshape(1, 1, -1), out[:, 1:]], dim=1)


def _moment_scale(f):
    z, w = np.polynomial.hermite_e.hermegauss(200)
    w = w / math.sqrt(2 * math.pi)
    fz = f(torch.tensor(z, dtype=torch.float64)).numpy()
    c = float(np.sum(w * fz * fz)) ** -0.5
    return 1.0 if abs(c - 1.0) < 1e-4 else c


C_SILU = _moment_scale(F.silu)
C_SIGMOID = _moment_scale(torch.sigmoid)


def ffn(p, pre, x, lmax):
    """mu:2694-2797: SO3 linear -> gate -> SO3 linear."""
    h = R.so3_linear(x, p[f"{pre}slinear_1.weight"], p[f"{pre}slinear_1.bias"])
    C = h.shape[-1]
    s = F.linear(h[:, 0:1], p[f"{pre}gate.gates.weight"], p[f"{pre}gate.gates.bias"])
    out = [F.silu(s[:, :, :C]) * C_SILU]
    start = 1
    for l in range(1, lmax + 1):
        out.append(torch.sigmoid(s[:, :, l * C:(l + 1) * C]) * C_SIGMOID * h[:, start:start + 2 * l + 1])
        start += 2 * l + 1
    h = torch.cat(out, dim=1)
    return R.so3_linear(h, p[f"{pre}slinear_2.weight"], p[f"{pre}slinear_2.bias"])


def spherical_harmonics(v):
    """Component-normalised real spherical harmonics l <= 2 of unit vectors, e3nn order: [E, 9]."""
    x, y, z = v[:, 0], v[:, 1], v[:, 2]
    s3, s5, s15 = math.sqrt(3.0), math.sqrt(5.0), math.sqrt(15.0)
    return torch.stack([torch.ones_like(x), s3 * x, s3 * y, s3 * z, s15 * x * z, s15 * x * y,
                        s5 * (y * y - 0.5 * (x * x + z * z)), s15 * y * z, 0.5 * s15 * (z * z - x * x)], dim=-1)


def edge_degree_embedding(p, pre, rbf, Z, qi, ni, outcell, edge_vec, poly, n_nodes, lmax, avg_degree):
    """e2f/e2former.py:689-753 with ``use_atom_edge``."""
    tgt = p[f"{pre}target_embedding.weight"][Z]
    src = p[f"{pre}source_embedding.weight"][Z][outcell]
    x_edge = torch.cat([rbf, tgt[qi], src[ni]], dim=-1)
    sh = spherical_harmonics(F.normalize(edge_vec, dim=-1))
    feats = []
    for l in range(lmax + 1):
        fea = R._mlp(x_edge, p, f"{pre}gbf_projs.{l}.net", 3) * poly.reshape(-1, 1)
        feats.append(R.edge_outer(sh[:, l * l:(l + 1) ** 2], fea, qi, n_nodes))
    return torch.cat(feats, dim=1) / avg_degree


def _y_rot(angle, l):
    """mu:275-302"""
    M = angle.new_zeros(angle.shape + (2 * l + 1, 2 * l + 1))
    for i, f in enumerate(range(l, -l - 1, -1)):
        M[..., i, 2 * l - i] = torch.sin(f * angle)
        M[..., i, i] = torch.cos(f * angle)
    return M


def wigner(pos, jd, l3_sequential, eps=1e-5):
    """mu:182-226 (eval: gamma = 0; pole / origin entries detached) and mu:305-337."""
    p = pos.to(torch.float64)
    d = torch.norm(p, dim=1)
    small = d < eps
    d = torch.where(small, torch.ones_like(d), d)
    xyz = p / d.view(-1, 1)
    y = xyz[:, 1]
    mask = small | torch.isclose(y.abs(), torch.ones_like(y))
    y_safe = torch.where(mask, torch.zeros_like(y), y)
    beta = torch.where(mask, torch.acos(y).detach(), torch.acos(y_safe))
    xs = torch.where(mask, torch.ones_like(y), xyz[:, 0])
    zs = torch.where(mask, torch.ones_like(y), xyz[:, 2])
    alpha = torch.where(mask, torch.atan2(xyz[:, 0], xyz[:, 2]).detach(), torch.atan2(xs, zs))
    a, b, c = torch.zeros_like(alpha), -beta, -alpha
    blocks = [_y_rot(a, l) @ jd[l] @ _y_rot(b, l) @ jd[l] @ _y_rot(c, l) for l in range(len(jd))]
    n = p.shape[0]
    size = sum(bk.shape[-1] for bk in blocks)
    W = p.new_zeros((n, size, size))
    s = 0
    for bk in blocks:
        W[:, s:s + bk.shape[-1], s:s + bk.shape[-1]] = bk
        s += bk.shape[-1]
    S = sum((2 * l + 1) * cnt for l, cnt in l3_sequential)
    Wi = p.new_zeros((n, S, S))
    s = 0
    for l, cnt in l3_sequential:
        for _ in range(cnt):
            Wi[:, s:s + 2 * l + 1, s:s + 2 * l + 1] = blocks[l]
            s += 2 * l + 1
    # the reference casts to fp32 for its fp32 model; a float64 caller (second-order checks) keeps float64
    out = torch.float64 if pos.dtype == torch.float64 else torch.float32
    return W.to(out), Wi.transpose(1, 2).contiguous().to(out)


def gaussian_rbf(dist, nb, cutoff):
    """mu:1853-1870 (basis width 2)."""
    offset = torch.linspace(0, cutoff, nb)
    coeff = -0.5 / (2.0 * (offset[1] - offset[0])).item() ** 2
    return torch.exp(coeff * (dist.view(-1, 1) - offset.view(1, -1)) ** 2)


def polynomial(dist, cutoff, p=5):
    """mu:1946-1954"""
    a, b, c = -(p + 1) * (p + 2) / 2, p * (p + 2), -p * (p + 1) / 2
    r = dist / cutoff
    return torch.where(r < 1, 1 + r ** p * (a + r * (b + c * r)), torch.zeros_like(r))


def system_embedding(p, charge, multiplicity):
    """e2f/e2former_wrapper.py:249-255: SiLU(Linear([emb_q(clip(q,-10,10)+10), emb_s(clip(s,0,20))]))
    per system, [B, C]; ``p`` holds the backbone-level parameters (``embedding_charge.weight`` ...)."""
    q = torch.clamp(torch.as_tensor(charge).reshape(-1).long(), -10, 10) + 10
    s = torch.clamp(torch.as_tensor(multiplicity).reshape(-1).long(), 0, 20)
    h = torch.cat([p["embedding_charge.weight"][q], p["embedding_multiplicity.weight"][s]], dim=-1)
    return F.silu(F.linear(h, p["mix_cm.0.weight"], p["mix_cm.0.bias"]))


def backbone(p, cfg, pos, Z, qi, ni, outcell, exp_pos, pbc_any, sys_node=None):
    """e2f/e2former.py:944-1145 (no cluster blocks) -> node irreps [N, 9, C].  ``sys_node`` [N, C]: the
    system embedding of each atom's system, added to the normed l=0 row of every block (582-583)."""
    lmax, nb, cutoff = 2, cfg["number_of_basis"], cfg["max_radius"]
    H, D = cfg["num_attn_heads"], cfg["attn_scalar_head"]
    l3 = R.L3_SEQUENTIAL
    jd = [p[f"Jd_list.{l}"].double() for l in range(lmax + 1)]
    W, Wi = wigner(pos, jd, l3)
    We, Wie = wigner(exp_pos, jd, l3) if pbc_any else (W, Wi)
    vec = pos[qi] - exp_pos[ni]
    dist = torch.linalg.norm(vec, dim=-1)
    poly = polynomial(dist, cutoff)
    rbf = gaussian_rbf(dist, nb, cutoff)
    x = edge_degree_embedding(p, "edge_deg_embed_dense.", rbf, Z, qi, ni, outcell, vec, poly, pos.shape[0], lmax,
                              cfg.get("avg_degree", 23.01))
    bd = {"query_idx": qi, "neighbor_idx": ni, "f_outcell_index": outcell, "f_exp_node_pos": exp_pos,
          "wigner": W, "wigner_inv": Wi, "wigner_exp": We, "wigner_inv_exp": Wie}
    for i in range(cfg["num_layers"]):
        pre = f"blocks.{i}."
        res = x
        h = rms_norm(p, pre + "norm_1.", x, lmax)
        if sys_node is not None:
            h = torch.cat([h[:, :1] + sys_node.unsqueeze(1), h[:, 1:]], dim=1)
        h = R.attention_layer(_sub(p, pre + "ga."), H, D, pos, h, dist, rbf, Z, poly, bd)
        x = h + res
        x = x + ffn(p, pre + "ffn.", rms_norm(p, pre + "norm_ffn.", x, lmax), lmax)
    return rms_norm(p, "norm_final.", x, lmax)


def energy_forces(p_backbone, p_head, cfg, pos, Z, graph, batch=None, p_system=None, charge=None,
                  multiplicity=None):
    """Energies per system and forces -dE/dpos.  ``graph`` = (qi, ni, outcell, image offsets [N2,3]
    or None, pbc_any): expanded positions are pos[outcell] + offset, so forces include the images.
    With ``charge`` given, ``p_system`` holds the backbone-level parameters of :func:`system_embedding`."""
    qi, ni, outcell, offsets, pbc_any = graph
    pos = pos.detach().clone().requires_grad_(True)
    exp_pos = pos[outcell] + offsets if offsets is not None else pos[outcell]
    sys_node = None
    if charge is not None:
        se = system_embedding(p_system, charge, multiplicity)
        sys_node = se[batch] if batch is not None else se[:1].expand(pos.shape[0], -1)
    x = backbone(p_backbone, cfg, pos, Z, qi, ni, outcell, exp_pos, pbc_any, sys_node)
    h = F.silu(F.linear(x[:, 0], p_head["mlp.0.weight"], p_head["mlp.0.bias"]))
    h = F.silu(F.linear(h, p_head["mlp.2.weight"], p_head["mlp.2.bias"]))
    e_atom = F.linear(h, p_head["mlp.4.weight"], p_head["mlp.4.bias"]).squeeze(-1)
    if batch is None:
        energy = e_atom.sum().reshape(1)
    else:
        energy = torch.zeros(int(batch.max()) + 1, dtype=e_atom.dtype).index_add(0, batch, e_atom)
    (g,) = torch.autograd.grad(energy.sum(), pos)
    return energy.detach(), -g, x.detach()
