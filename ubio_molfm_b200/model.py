"""E2Former-V2 backbone and energy / force evaluation on top of the B200 attention layer.

Mirrors, with the same parameter names (so reference checkpoints load by name):

* ``EquivariantRMSNormArraySphericalHarmonicsV2_BL`` -- module_utils.py:1663-1772;
* ``Gate_s3`` / ``FeedForwardNetwork_s3``           -- module_utils.py:2694-2797;
* ``TransBlock``                                     -- e2former.py:440-620 (pre-norm attention + FFN);
* ``EdgeDegreeEmbeddingNetwork_higherorder``         -- e2former.py:623-753;
* ``E2former``                                       -- e2former.py:756-1145 (no ``with_cluster`` blocks);
* ``MLP_energy_head`` and the autograd force head    -- pipeline/head.py:305-345.

``E2FormerPotential`` is the whole evaluation the ASE / MD interfaces call: CUDA PBC images and
radius graph, per-node Wigner matrices, the backbone, per-atom energies summed per system and
forces = -dE/dpos by autograd through the graph geometry.
"""
from __future__ import annotations

import math

import numpy as np
import torch
from torch import nn

from . import _lib
from . import linear as tc
from . import ops
from .attention import E2AttentionArbOrder_sparse
from .graph import distributed_cell_expand, expand_pbc, radius_graph
from .nn import GaussianSmearing, RadialProfile, RbfSpec, SO3_Linear_e2former, irreps_channels_lmax, lin, run_mlp
from .wigner import jd_matrices, node_wigner


# ------------------------------------------------------------------------------------------------
# a8: equivariant RMS norm
# ------------------------------------------------------------------------------------------------
class EquivariantRMSNormArraySphericalHarmonicsV2_BL(nn.Module):
    """Centre the l=0 row over channels, divide every row by the degree-balanced RMS over all (m, c)
    of the node, scale per degree, add a bias on l=0 (module_utils.py:1663-1772, component
    normalisation with ``std_balance_degrees``)."""

    def __init__(self, lmax, num_channels, eps=1e-5, affine=True, normalization="component", centering=True,
                 std_balance_degrees=True):
        super().__init__()
        if normalization != "component" or not affine or not centering or not std_balance_degrees:
            raise NotImplementedError("only the default (component, affine, centred, balanced) norm is built")
        self.lmax, self.num_channels, self.eps = lmax, num_channels, eps
        self.affine_weight = nn.Parameter(torch.ones(lmax + 1, num_channels))
        self.affine_bias = nn.Parameter(torch.zeros(num_channels))
        idx = torch.tensor([l for l in range(lmax + 1) for _ in range(2 * l + 1)], dtype=torch.long)
        self.register_buffer("expand_index", idx)
        bw = torch.tensor([1.0 / (2 * l + 1) for l in range(lmax + 1) for _ in range(2 * l + 1)]) / (lmax + 1)
        self.register_buffer("balance_degree_weight", bw.reshape(-1, 1))

    def forward(self, x, batch=None):
        shape = x.shape
        f = x.reshape(-1, (self.lmax + 1) ** 2, self.num_channels)
        if not self.training and tc.rms_norm_supported(f):
            return tc.rms_norm(f, self.affine_weight, self.affine_bias, self.eps).reshape(shape)
        f0 = f[:, :1] - f[:, :1].mean(dim=2, keepdim=True)
        f = torch.cat([f0, f[:, 1:]], dim=1)
        ms = (f.pow(2) * self.balance_degree_weight.reshape(1, -1, 1)).sum(dim=1, keepdim=True)
        scale = (ms.mean(dim=2, keepdim=True) + self.eps).pow(-0.5)
        out = f * (scale * self.affine_weight[self.expand_index].unsqueeze(0))
        out = torch.cat([out[:, :1] + self.affine_bias.reshape(1, 1, -1), out[:, 1:]], dim=1)
        return out.reshape(shape)


def get_normalization_layer(norm_type, lmax, num_channels, eps=1e-5, affine=True, normalization="component"):
    """module_utils.py:1277-1297 (the two kinds this build has)."""
    if norm_type in ("rms_norm_sh", "rms_norm_sh_BL"):
        return EquivariantRMSNormArraySphericalHarmonicsV2_BL(lmax, num_channels, eps, affine, normalization)
    if norm_type == "identity":
        return nn.Identity()
    raise NotImplementedError(f"norm_layer={norm_type!r}")


# ------------------------------------------------------------------------------------------------
# a17: gated feed-forward network and the transformer block
# ------------------------------------------------------------------------------------------------
def second_moment_scale(f, n=200):
    """1 / sqrt(E[f(z)^2]) for z ~ N(0, 1) by probabilists' Gauss-Hermite quadrature (the second-moment
    normaliser of an activation, e3nn.math.normalize2mom); 1.0 when already within 1e-4 of one."""
    z, w = np.polynomial.hermite_e.hermegauss(n)
    w = w / math.sqrt(2 * math.pi)
    with torch.no_grad():
        fz = f(torch.tensor(z, dtype=torch.float64)).numpy()
    c = float(np.sum(w * fz * fz)) ** -0.5
    return 1.0 if abs(c - 1.0) < 1e-4 else c


class Gate_s3(nn.Module):
    """Scalars -> normalised SiLU; degree l > 0 rows scaled by a normalised sigmoid of their own gate
    channels, all gates from one linear of the l=0 row (module_utils.py:2694-2745)."""

    def __init__(self, sphere_channels, lmax, act_scalars="silu", act_vector="sigmoid"):
        super().__init__()
        if act_scalars != "silu" or act_vector != "sigmoid":
            raise NotImplementedError("Gate_s3 supports silu scalars and sigmoid gates")
        self.sphere_channels, self.lmax = sphere_channels, lmax
        self.gates = nn.Linear(sphere_channels, sphere_channels * (lmax + 1))
        bound = 1 / math.sqrt(sphere_channels)
        nn.init.uniform_(self.gates.weight, -bound, bound)
        self.c_silu = second_moment_scale(torch.nn.functional.silu)
        self.c_sigmoid = second_moment_scale(torch.sigmoid)

    def forward(self, x):
        shape = x.shape
        x = x.reshape(-1, shape[-2], shape[-1])
        C = self.sphere_channels
        s = lin(x[:, 0], self.gates.weight, self.gates.bias, not self.training)       # [n, C (lmax+1)]
        if x.is_cuda and not self.training and self.lmax == 2 and C % 4 == 0:
            return tc.gate(s, x, self.c_silu, self.c_sigmoid).reshape(shape)
        out = [(torch.nn.functional.silu(s[:, :C]) * self.c_silu).unsqueeze(1)]
        start = 1
        for l in range(1, self.lmax + 1):
            g = torch.sigmoid(s[:, l * C:(l + 1) * C]) * self.c_sigmoid
            out.append(g.unsqueeze(1) * x[:, start:start + 2 * l + 1])
            start += 2 * l + 1
        return torch.cat(out, dim=1).reshape(shape)


class FeedForwardNetwork_s3(nn.Module):
    """SO3 linear -> gate -> SO3 linear (module_utils.py:2748-2797)."""

    def __init__(self, sphere_channels, hidden_channels, output_channels, lmax):
        super().__init__()
        self.slinear_1 = SO3_Linear_e2former(sphere_channels, hidden_channels, lmax=lmax, bias=True)
        self.gate = Gate_s3(hidden_channels, lmax=lmax)
        self.slinear_2 = SO3_Linear_e2former(hidden_channels, output_channels, lmax=lmax, bias=True)

    def forward(self, x, **kwargs):
        return self.slinear_2(self.gate(self.slinear_1(x)))


class TransBlock(nn.Module):
    """Pre-norm residual attention + pre-norm residual gated FFN (e2former.py:440-620)."""

    def __init__(self, irreps_node_input="256x0e+256x1e+256x2e", irreps_node_output="256x0e+256x1e+256x2e",
                 attn_weight_input_dim=32, num_attn_heads=8, attn_scalar_head=32, irreps_head="32x0e+32x1e+32x2e",
                 alpha_drop=0.1, tp_type="QK_alpha", attn_type="first-order", atom_type_cnt=256,
                 norm_layer="identity", ffn_type="s3", layer_id=0):
        super().__init__()
        C, lmax = irreps_channels_lmax(irreps_node_input)
        self.lmax = lmax
        self.norm_1 = get_normalization_layer(norm_layer, lmax=lmax, num_channels=C)
        self.ga = E2AttentionArbOrder_sparse(irreps_node_input, attn_weight_input_dim, num_attn_heads,
                                             attn_scalar_head, irreps_head, alpha_drop=alpha_drop,
                                             attn_type=attn_type, tp_type=tp_type, norm_layer=norm_layer,
                                             atom_type_cnt=atom_type_cnt)
        if "default" not in ffn_type and "s3" not in ffn_type:
            raise NotImplementedError(f"ffn_type={ffn_type!r}")
        self.norm_ffn = get_normalization_layer(norm_layer, lmax=lmax, num_channels=C)
        self.ffn = FeedForwardNetwork_s3(C, C, C, lmax=lmax)

    def forward(self, node_pos, node_irreps, sys_node_embedding, edge_dis, edge_vec, attn_weight, atomic_numbers,
                attn_mask, poly_dist=None, batch=None, batched_data=None, **kwargs):
        node_irreps = node_irreps[:, :(self.lmax + 1) ** 2]
        # rows past n_query (domain ghosts) only serve as keys / values: the block returns the query rows
        nq = int(batched_data.get("n_query", node_irreps.shape[0])) if batched_data is not None else node_irreps.shape[0]
        res = node_irreps[:nq]
        h = self.norm_1(node_irreps)
        if sys_node_embedding is not None:
            h = torch.cat([h[:, :1] + sys_node_embedding.unsqueeze(1), h[:, 1:]], dim=1)
        h, attn_weight = self.ga(node_pos=node_pos, node_irreps_input=h, edge_dis=edge_dis, poly_dist=poly_dist,
                                 edge_vec=edge_vec, attn_weight=attn_weight, atomic_numbers=atomic_numbers,
                                 attn_mask=attn_mask, batched_data=batched_data)
        h = h + res
        return h + self.ffn(self.norm_ffn(h)), attn_weight


# ------------------------------------------------------------------------------------------------
# a7: initial irreps from the edge-degree embedding
# ------------------------------------------------------------------------------------------------
def spherical_harmonics_l2(v):
    """Real spherical harmonics of unit vectors up to l = 2, component normalisation, in the order and
    axis convention of e3nn's ``_spherical_harmonics`` (y is the polar axis): [E, 9]."""
    x, y, z = v[:, 0], v[:, 1], v[:, 2]
    s3, s5, s15 = math.sqrt(3.0), math.sqrt(5.0), math.sqrt(15.0)
    return torch.stack([torch.ones_like(x), s3 * x, s3 * y, s3 * z, s15 * x * z, s15 * x * y,
                        s5 * (y * y - 0.5 * (x * x + z * z)), s15 * y * z, 0.5 * s15 * (z * z - x * x)], dim=-1)


class EdgeDegreeEmbeddingNetwork_higherorder(nn.Module):
    """x[n, l-block, c] = sum_e SH_l(v_e) (MLP_l([rbf, embT(Z_i), embS(Z_j)]) poly_e)_c / avg_degree
    (e2former.py:623-753; ``use_atom_edge``).  The first linear of each MLP is split exactly into an RBF
    product plus per-element tables, as in the attention's radial MLP."""

    def __init__(self, irreps_node_embedding, avg_aggregate_num=10, number_of_basis=32, cutoff=15,
                 time_embed=False, use_layer_norm=True, use_atom_edge=False, name="default", **kwargs):
        super().__init__()
        if time_embed:
            raise NotImplementedError("time embedding is a training-only option")
        C, lmax = irreps_channels_lmax(irreps_node_embedding)
        self.cutoff, self.number_of_basis, self.scalar_dim, self.lmax = cutoff, number_of_basis, C, lmax
        self.max_num_elements = 300
        self.use_atom_edge = use_atom_edge
        if use_atom_edge:
            self.source_embedding = nn.Embedding(self.max_num_elements, number_of_basis)
            self.target_embedding = nn.Embedding(self.max_num_elements, number_of_basis)
        else:
            self.source_embedding = None
            self.target_embedding = None
        hid = min(number_of_basis // 2, 128)
        self.gbf_projs = nn.ModuleList([
            RadialProfile([number_of_basis * 3 if use_atom_edge else number_of_basis, hid, hid, C],
                          use_layer_norm=use_layer_norm) for _ in range(lmax + 1)])
        self.proj = SO3_Linear_e2former(C * 2, C, lmax=lmax)   # present in checkpoints; unused by forward
        self.avg_aggregate_num = avg_aggregate_num
        self.name = name

    def forward(self, node_input, node_pos, edge_dis, atomic_numbers, edge_vec, batched_data, attn_mask, poly_dist,
                edge_scalars, **kwargs):
        qi = batched_data["query_idx"].to(torch.long)
        ni = batched_data["neighbor_idx"].to(torch.long)
        n = int(batched_data.get("n_query", node_pos.shape[0]))   # output rows: the query rows
        nb = self.number_of_basis
        cw = not self.training
        sh = spherical_harmonics_l2(torch.nn.functional.normalize(edge_vec, dim=-1))
        feats = []
        for l, prof in enumerate(self.gbf_projs):
            layers = list(prof.net)
            lin0 = layers[0]
            w = lin0.weight.detach() if cw else lin0.weight
            if self.use_atom_edge:
                with torch.set_grad_enabled(torch.is_grad_enabled() and not cw):
                    t_tab = (self.target_embedding.weight @ w[:, nb:2 * nb].t()).contiguous()
                    s_tab = (self.source_embedding.weight @ w[:, 2 * nb:].t()).contiguous()
                z_q = atomic_numbers[qi]
                z_k = atomic_numbers[batched_data["f_outcell_index"]][ni]
                if isinstance(edge_scalars, RbfSpec):
                    h = edge_scalars.linear(w[:, :nb], lin0.bias, cw)
                else:
                    h = lin(edge_scalars, w[:, :nb], lin0.bias, cw)
                h = run_mlp(layers[1:], h, cw, first_tables=(t_tab, z_q, s_tab, z_k))
            else:
                h = prof(edge_scalars.materialize() if isinstance(edge_scalars, RbfSpec) else edge_scalars)
            # the envelope scales each edge's product: applied to the [E, 2l+1] harmonics rather than the
            # [E, C] features (the same sum, a fraction of the elementwise work)
            sh_l = sh[:, l * l:(l + 1) ** 2] * poly_dist.reshape(-1, 1)
            feats.append(ops.edge_degree_outer_triton(sh_l.contiguous(), h.contiguous(), qi, n,
                                                      batched_data["metadata"]))
        return torch.cat(feats, dim=1) / self.avg_aggregate_num


# ------------------------------------------------------------------------------------------------
# a18: the backbone and the heads
# ------------------------------------------------------------------------------------------------
class E2former(nn.Module):
    """Edge-degree embedding -> ``num_layers`` TransBlocks -> final norm (e2former.py:756-1145)."""

    def __init__(self, irreps_node_embedding="128x0e+128x1e+128x2e", num_layers=6, max_neighbors=300,
                 max_radius=4.5, basis_type="gaussiansmear", number_of_basis=128, num_attn_heads=4,
                 attn_scalar_head=32, irreps_head="32x0e+32x1e+32x2e", norm_layer="rms_norm_sh", alpha_drop=0.1,
                 tp_type="QK_alpha", attn_type="first-order", atom_type_cnt=256, edge_embedtype="default",
                 ffn_type="default", avg_degree=23.01, with_cluster=False, **kwargs):
        super().__init__()
        if str(with_cluster) not in {"False", "false", "0", "None", "none"}:
            raise NotImplementedError("with_cluster long-range blocks are not built")
        if basis_type != "gaussiansmear":
            raise NotImplementedError(f"basis_type={basis_type!r}")
        C, lmax = irreps_channels_lmax(irreps_node_embedding)
        self.irreps_node_embedding = irreps_node_embedding
        self.max_neighbors, self.max_radius, self.number_of_basis = max_neighbors, max_radius, number_of_basis
        self.num_layers, self.lmax, self.scalar_dim = num_layers, lmax, C
        self._node_scalar_dim = C
        attn_types = attn_type.split("+") if "+" in attn_type else [attn_type, attn_type]
        self.default_node_embedding = nn.Embedding(atom_type_cnt, C)
        self.heads2basis = nn.Linear(num_attn_heads, number_of_basis, bias=True)   # present in checkpoints
        self.rbf = GaussianSmearing(number_of_basis, cutoff=max_radius, basis_width_scalar=2)
        self.Jd_list = nn.ParameterList([nn.Parameter(j.float(), requires_grad=False) for j in jd_matrices(lmax)])
        self.edge_deg_embed_dense = EdgeDegreeEmbeddingNetwork_higherorder(
            irreps_node_embedding, avg_degree, cutoff=max_radius, number_of_basis=number_of_basis,
            use_atom_edge=True, use_layer_norm="wolayernorm" not in edge_embedtype)
        self.blocks = nn.ModuleList([
            TransBlock(irreps_node_embedding, irreps_node_embedding, attn_weight_input_dim=number_of_basis,
                       num_attn_heads=num_attn_heads, attn_scalar_head=attn_scalar_head, irreps_head=irreps_head,
                       alpha_drop=alpha_drop, tp_type=tp_type,
                       attn_type=attn_types[0] if i < num_layers // 2 else attn_types[1], norm_layer=norm_layer,
                       ffn_type=ffn_type, layer_id=i, atom_type_cnt=atom_type_cnt)
            for i in range(num_layers)])
        self.l3_sequential = self.blocks[0].ga.first_order_tp.so2_tp.l3_sequential
        self.norm_final = get_normalization_layer(norm_layer, lmax=lmax, num_channels=C)
        self._register_load_state_dict_pre_hook(self._drop_unused_constants)

    def _drop_unused_constants(self, state_dict, prefix, *args):
        """Reference checkpoints also carry the J matrices of degrees above lmax (Jd.pt holds l <= 11)
        and the l=2 harmonic coefficient table of an unused module (``sph_fromxyz``): constants this
        model does not read.  They are dropped on load so strict loading works."""
        for k in list(state_dict.keys()):
            if not k.startswith(prefix):
                continue
            rest = k[len(prefix):]
            if rest.startswith("Jd_list.") and int(rest.split(".")[1]) > self.lmax:
                del state_dict[k]
            elif rest == "edge_deg_embed_dense.sph.W":
                del state_dict[k]

    def forward(self, node_pos, atomic_numbers, graph, pbc_any, halo=None, sys_embedding=None, kv_halo=None):
        """``graph``: the flattened neighbour dict (``query_idx``, ``neighbor_idx``, ``metadata``,
        ``f_edge_vec``, ``f_dist``, ``f_poly_dist``, ``f_outcell_index``, ``f_exp_node_pos`` and the
        optional ``row_order`` / ``key_order``).  Returns the node irreps [N, (lmax+1)^2, C].
        ``halo`` (domain decomposition): called on the node irreps before every block to refresh the
        rows of atoms owned by other ranks.  With ``graph["n_query"]`` = n, only rows [0, n) are queries:
        the embedding and every block return those rows, and ``halo`` appends the others before each
        block (it receives the n query rows).  ``sys_embedding`` ([rows, C] or [1, C], or None): the
        charge / multiplicity embedding of each row's system, added to the normed l=0 row of every
        block (e2former.py:1074-1077, 582-583); with a halo it must cover the appended rows too.
        ``kv_halo`` (domain decomposition, instead of ``halo``): the node irreps stay at the n query rows
        through every block, and each attention layer calls ``kv_halo(t, "key")`` / ``kv_halo(t, "value")``
        on its key / value projections of those rows, which must return them followed by the other
        atoms' projections (from their owners): no norm or projection work for rows owned elsewhere."""
        if int(graph.get("n_query", node_pos.shape[0])) != node_pos.shape[0] and halo is None and kv_halo is None:
            raise ValueError("n_query < number of nodes needs a halo to refresh the other rows")
        if halo is not None and kv_halo is not None:
            raise ValueError("pass halo or kv_halo, not both")
        jd = [j.to(torch.float64) for j in self.Jd_list]
        bd = dict(graph)
        if kv_halo is not None:
            bd["kv_halo"] = kv_halo
        if node_pos.is_cuda and not self.training and self.lmax == 2:
            # the attention layers form their per-node SO(2) maps from the positions directly
            bd.update({"wigner": None, "wigner_inv": None, "wigner_exp": None, "wigner_inv_exp": None,
                       "node_map_jd": list(self.Jd_list)})
        else:
            W, Wi = node_wigner(node_pos, self.lmax, self.l3_sequential, dtype=node_pos.dtype, jd=jd)
            if pbc_any:
                We, Wie = node_wigner(graph["f_exp_node_pos"], self.lmax, self.l3_sequential,
                                      dtype=node_pos.dtype, jd=jd)
            else:
                We, Wie = W, Wi
            bd.update({"wigner": W, "wigner_inv": Wi, "wigner_exp": We, "wigner_inv_exp": Wie})
        if node_pos.is_cuda and not self.training:
            # the basis is formed inside each consumer's first product (see linear.rbf_linear)
            f_dist_embedding = RbfSpec(graph["f_dist"], self.rbf.offset, self.rbf.coeff)
        else:
            f_dist_embedding = self.rbf(graph["f_dist"])
        x = self.edge_deg_embed_dense(node_input=None, node_pos=node_pos, edge_dis=graph["f_dist"],
                                      atomic_numbers=atomic_numbers, edge_vec=graph["f_edge_vec"], batched_data=bd,
                                      attn_mask=None, poly_dist=graph["f_poly_dist"], edge_scalars=f_dist_embedding)
        for blk in self.blocks:
            if halo is not None:
                x = halo(x)
            x, f_dist_embedding = blk(node_pos=node_pos, node_irreps=x, sys_node_embedding=sys_embedding,
                                      edge_dis=graph["f_dist"], edge_vec=graph["f_edge_vec"],
                                      attn_weight=f_dist_embedding, atomic_numbers=atomic_numbers, attn_mask=None,
                                      poly_dist=graph["f_poly_dist"], batched_data=bd)
        return self.norm_final(x)


class E2FormerBackbone(nn.Module):
    """The wrapper around :class:`E2former` with the reference's parameters and names
    (e2former_wrapper.py:36-339): the atom-type table ``embedding``, the system embedding of the total
    charge and spin multiplicity (``embedding_charge``, ``embedding_multiplicity``, ``mix_cm``),
    ``unifiedtokentoembedding`` and, with ``encoder != "default"``, ``embed_proj``; the decoder is
    ``self.decoder``.  A strict ``load_state_dict`` of the reference backbone's state dict works.

    Of these only the system embedding reaches the output: the decoder never reads the per-atom token
    embedding (e2former.py:1032-1043 passes it to the edge-degree embedding, which uses only its row
    count), so ``embedding`` / ``unifiedtokentoembedding`` / ``embed_proj`` are kept for checkpoints."""

    def __init__(self, use_faiss=False, **kwargs):
        super().__init__()
        self.use_faiss = use_faiss
        C, _ = irreps_channels_lmax(kwargs["irreps_node_embedding"])
        encoder = kwargs.get("encoder", "default")
        dim = C if encoder == "default" else kwargs["encoder_embed_dim"]
        self.embedding = nn.Embedding(256, dim)
        self.embedding_charge = nn.Embedding(30, dim)
        self.embedding_multiplicity = nn.Embedding(30, dim)
        self.mix_cm = nn.Sequential(nn.Linear(2 * dim, dim), nn.SiLU())
        self.unifiedtokentoembedding = nn.Linear(dim, dim)
        if encoder != "default":
            self.embed_proj = nn.Sequential(nn.Linear(kwargs["encoder_embed_dim"], C), nn.SiLU(),
                                            nn.LayerNorm(C, eps=1e-6))
        if kwargs.get("max_neighbors", None) == "None":
            kwargs["max_neighbors"] = None
        self.decoder = E2former(**kwargs)

    def system_embedding(self, charge, multiplicity):
        """[B, C] from the per-system total charge and spin multiplicity (integers, any shape holding
        B values): ``mix_cm([embedding_charge(clip(q, -10, 10) + 10), embedding_multiplicity(clip(m, 0,
        20))])`` (e2former_wrapper.py:249-255)."""
        q = torch.clamp(torch.as_tensor(charge).reshape(-1).to(torch.long), -10, 10) + 10
        s = torch.clamp(torch.as_tensor(multiplicity).reshape(-1).to(torch.long), 0, 20)
        dev = self.embedding_charge.weight.device
        h = torch.cat([self.embedding_charge(q.to(dev)), self.embedding_multiplicity(s.to(dev))], dim=-1)
        lin0 = self.mix_cm[0]
        return torch.nn.functional.silu(lin(h, lin0.weight, lin0.bias, not self.training))


class MLP_energy_head(nn.Module):
    """Per-atom energy from the l=0 features: Linear-SiLU-Linear-SiLU-Linear (pipeline/head.py:330-341)."""

    def __init__(self, embedding_dim, lmax=2):
        super().__init__()
        self.mlp = nn.Sequential(nn.Linear(embedding_dim, embedding_dim), nn.SiLU(),
                                 nn.Linear(embedding_dim, embedding_dim), nn.SiLU(), nn.Linear(embedding_dim, 1))

    def forward(self, embedding, irreps=None):
        cw = not self.training
        m = self.mlp
        h = torch.nn.functional.silu(lin(embedding, m[0].weight, m[0].bias, cw))
        h = torch.nn.functional.silu(lin(h, m[2].weight, m[2].bias, cw))
        return lin(h, m[4].weight, m[4].bias, cw)


class E2FormerPotential(nn.Module):
    """Energy + forces of one or more systems: CUDA graph build, backbone, per-atom energy head,
    forces = -dE/dpos (the GradientHead of pipeline/head.py:305-328).

    ``forward(pos [N,3], atomic_numbers [N], cell [3,3] or None, pbc (3 bools), batch [N] or None)`` ->
    ``(energy [B], forces [N,3])``.  Periodic systems are one per call; non-periodic molecules may be
    batched (``batch`` sorted, systems do not see each other)."""

    def __init__(self, memory_saving="auto", use_faiss=False, edge_chunk=None, **backbone_kwargs):
        super().__init__()
        # use_faiss: expanded nodes in the order of the reference's FAISS neighbour path
        # (distributed_cell_expand, one image cell per direction) instead of CellExpander's; the edges
        # are the same physical neighbours, found by the same exact search (FAISS itself is not used)
        self.use_faiss = use_faiss
        # after every evaluation, read (one stream sync) and clear the status word of the GEMM's bounded
        # waits, raising if one gave up: an aborted projection leaves its output partly unwritten
        self.check_device_status = True
        self.backbone = E2FormerBackbone(use_faiss=use_faiss, **backbone_kwargs)
        self.energy_head = MLP_energy_head(self.decoder.scalar_dim, self.decoder.lmax)
        # memory_saving: True = the Q / K per-degree projections are formed again in the backward instead
        # of kept (2 x heads x head-dim floats per irreps row and layer, ~29 GB at 1e5 atoms with the
        # full-size model; ~10% of the step's tensor-core work) and the attention span's q.k scores are
        # not kept (heads floats per edge and layer, ~6.4 GB at 1e5 atoms); False = both kept; "auto" =
        # both kept unless the evaluation's estimated peak passes 85% of the device's memory, then the
        # scores are dropped first, the projections second, and last the edge side runs in checkpointed
        # blocks of rows (``edge_chunk``, below)
        # edge_chunk: a number of edges; every attention layer then runs its radial MLP and span over
        # blocks of query rows of about that many edges, each checkpointed, so no [edges, .] tensor of
        # the whole graph is kept (eval mode; the backward forms each block's again)
        self.memory_saving = memory_saving
        self.edge_chunk = edge_chunk
        self._set_memory_mode(memory_saving is True, memory_saving is not True, edge_chunk)

    def _set_memory_mode(self, recompute, keep_logits, edge_chunk=None):
        for blk in self.decoder.blocks:
            blk.ga.query_linear.recompute_pair_product = recompute
            blk.ga.key_linear.recompute_pair_product = recompute
            blk.ga.keep_logits = keep_logits
            blk.ga.edge_chunk = edge_chunk

    # peak bytes of an evaluation per edge, projections recomputed and scores not kept (measured:
    # 112.6 GB at 3.13 M edges)
    _PEAK_BYTES_PER_EDGE = 36.0e3

    def _auto_memory_mode(self, n_rows, n_edges, device):
        """(recompute projections, keep scores, edge block) for a graph of this size
        (``memory_saving="auto"``)."""
        dec = self.decoder
        blk = dec.blocks[0].ga
        layers = len(dec.blocks)
        proj = 2 * layers * n_rows * (dec.lmax + 1) ** 2 * blk.num_attn_heads * blk.attn_scalar_head * 4
        logits = layers * n_edges * blk.num_attn_heads * 4
        base = self._PEAK_BYTES_PER_EDGE * n_edges
        cap = 0.85 * torch.cuda.get_device_properties(device).total_memory
        chunk = self.edge_chunk
        if base + proj + logits <= cap:
            return False, True, chunk
        if base + proj <= cap:
            return False, False, chunk
        if base <= cap:
            return True, False, chunk
        return True, False, chunk or self._AUTO_EDGE_CHUNK

    # edges per block when "auto" has to run the edge side in blocks
    _AUTO_EDGE_CHUNK = 4_000_000

    @property
    def decoder(self):
        """The :class:`E2former` inside the backbone."""
        return self.backbone.decoder

    def load_reference_state_dict(self, state_dict, head_name=None, strict=True):
        """Load a reference ``MolfmAtomic`` state dict (tasks/pretrain_smallmol.py:170-210): ``decoder.*``
        is the backbone, ``head.energy_heads.<head_name>.mlp.*`` the energy MLP.  With ``head_name``
        None the state dict must hold exactly one energy head."""
        sd = {}
        heads = sorted({k.split(".")[2] for k in state_dict if k.startswith("head.energy_heads.")})
        if head_name is None:
            if len(heads) != 1:
                raise ValueError(f"state dict holds energy heads {heads}: pass head_name")
            head_name = heads[0]
        elif head_name not in heads:
            raise KeyError(f"no energy head {head_name!r} in the state dict (has {heads})")
        pre = f"head.energy_heads.{head_name}."
        for k, v in state_dict.items():
            if k.startswith("decoder."):
                sd["backbone." + k[len("decoder."):]] = v
            elif k.startswith(pre):
                sd["energy_head." + k[len(pre):]] = v
        return self.load_state_dict(sd, strict=strict)

    def build_graph(self, pos, cell, pbc, batch):
        dec = self.decoder
        n = pos.shape[0]
        dev = pos.device
        pbc_any = bool(cell is not None and any(bool(p) for p in pbc))
        if pbc_any:
            if batch is not None and int(batch.max()) > 0:
                raise NotImplementedError("periodic systems are evaluated one per call")
            if self.use_faiss:
                pd = pos.detach()
                ex = distributed_cell_expand(pos.unsqueeze(0), torch.as_tensor(cell, dtype=torch.float32),
                                             dec.max_radius, pd.min(dim=0).values, pd.max(dim=0).values, 1,
                                             torch.as_tensor([bool(v) for v in pbc]))
                exp_pos, outcell = ex["expand_node_pos"][0], ex["outcell_index"][0]
            else:
                exp_pos, outcell, _ = expand_pbc(pos, torch.as_tensor(cell, dtype=torch.float32), list(pbc),
                                                 dec.max_radius)
            q_ptr = torch.tensor([0, n])
            p_ptr = torch.tensor([0, exp_pos.shape[0]])
        else:
            exp_pos = pos
            outcell = torch.arange(n, device=dev)
            if batch is None:
                q_ptr = torch.tensor([0, n])
            else:
                counts = torch.bincount(batch, minlength=int(batch.max()) + 1).cpu()
                q_ptr = torch.nn.functional.pad(counts.cumsum(0), (1, 0))
            p_ptr = q_ptr
        g = radius_graph(pos, exp_pos, q_ptr, p_ptr, dec.max_radius, 1e-4, dec.max_neighbors)
        g["f_outcell_index"] = outcell
        g["f_exp_node_pos"] = exp_pos
        return g, pbc_any

    def forward(self, pos, atomic_numbers, cell=None, pbc=(False, False, False), batch=None, need_forces=True,
                charge=None, multiplicity=None, create_graph=None):
        """``charge`` / ``multiplicity``: per-system integers ([B] or None).  Given (as the reference's
        interface always does, interface/data_utils.py:53-65), their system embedding is added to the
        normed l=0 row of every block; None evaluates the decoder without it (e2former_wrapper.py:249-250
        with no ``charge`` key).  ``multiplicity`` defaults to 1 when only ``charge`` is given.

        ``create_graph`` (default: ``self.training``, as pipeline/head.py:318-325 takes the force gradient):
        the forces keep their graph and the energy is not detached, so a loss on both can be
        back-propagated to the parameters (force-loss training; training mode only)."""
        if create_graph is None:
            create_graph = self.training and need_forces
        if create_graph and not self.training:
            raise RuntimeError("create_graph=True needs training mode (model.train()): the eval-mode fused "
                               "ops are first-order only")
        pos = pos.detach().to(torch.float32).requires_grad_(need_forces)
        with torch.enable_grad() if need_forces else torch.no_grad():
            g, pbc_any = self.build_graph(pos, cell, pbc, batch)
            if self.memory_saving == "auto" and pos.is_cuda:
                self._set_memory_mode(*self._auto_memory_mode(pos.shape[0], g["query_idx"].numel(), pos.device))
            sys_emb = None
            if charge is not None:
                if multiplicity is None:
                    multiplicity = torch.ones_like(torch.as_tensor(charge))
                sys_emb = self.backbone.system_embedding(charge, multiplicity)
                sys_emb = sys_emb[batch] if batch is not None else sys_emb[:1]
            x = self.decoder(pos, atomic_numbers, g, pbc_any, sys_embedding=sys_emb)
            e_atom = self.energy_head(x[:, 0]).squeeze(-1)
            if batch is None:
                energy = e_atom.sum().reshape(1)
            else:
                energy = torch.zeros(int(batch.max()) + 1, device=pos.device, dtype=e_atom.dtype)
                energy = energy.index_add(0, batch, e_atom)
            forces = None
            if need_forces:
                (grad,) = torch.autograd.grad(energy.sum(), pos, create_graph=create_graph)
                forces = -grad
        if pos.is_cuda and self.check_device_status:
            _lib.raise_on_device_status(pos.device)
        return (energy if create_graph else energy.detach()), forces
