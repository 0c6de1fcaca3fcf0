"""``E2AttentionArbOrder_sparse`` -- drop-in for the reference attention layer (e2former.py:80-436).

Same constructor arguments, parameter names (``state_dict`` keys) and ``forward`` signature as the
reference with ``tp_type="QK_alpha"`` (``"+triton"`` accepted and ignored) and
``attn_type="so2-first-order"`` / ``"first-order"``.  Per layer:

* node side (dense, cuBLAS): Q/K ``SO3_Linear2Scalar``, ``proj_value``, the two node-local halves
  of the first-order SO(2) tensor product with the per-node Wigner matrices, ``forward_linear``,
  ``proj_first``;
* edge side: the radial MLP ``fc_easy`` with its first layer decomposed exactly into an RBF part
  and per-element tables (no ``[E, nb+256]`` concatenation), then ONE fused CUDA kernel for
  QK logits -> gated segmented softmax -> alpha/r -> value aggregation (and two for its backward),
  which never materialises per-edge value tensors.
"""
from __future__ import annotations

import math

import torch
from torch import nn

from .nn import (E2TensorProductSO2_FirstOrder, RbfSpec, RadialProfile, SO3_Linear2Scalar_e2former, SO3_Linear_e2former,
                 irreps_channels_lmax, lin, parse_irreps, run_mlp)
from . import linear as tc
from .ops import attention_span


def edge_blocks(row_ptr, row_order, edge_chunk):
    """Split the query rows of a query-sorted CSR (``row_ptr`` [n+1]) into blocks of about ``edge_chunk``
    edges: consecutive runs of ``row_order`` (all rows once; None = index order).  Per block
    ``(rows, local, edges)``: its rows in that order, each of its edges' row position within the block
    (ascending), and the edges' ids, row by row in CSR order.  Device tensors; a few host reads."""
    row_ptr = row_ptr.to(torch.int64)
    n_rows = row_ptr.numel() - 1
    dev = row_ptr.device
    order = (torch.arange(n_rows, device=dev) if row_order is None or row_order.numel() != n_rows
             else row_order.to(torch.int64))
    E = int(row_ptr[-1])
    deg = (row_ptr[1:] - row_ptr[:-1])[order]
    csum = torch.cumsum(deg, 0)
    targets = torch.arange(1, max((E + edge_chunk - 1) // edge_chunk, 1), device=dev) * edge_chunk
    cuts = [0] + sorted(set(int(c) for c in torch.searchsorted(csum, targets).tolist() if 0 < int(c) < n_rows))
    cuts.append(n_rows)
    out = []
    for a, b in zip(cuts[:-1], cuts[1:]):
        rows = order[a:b]
        d = deg[a:b]
        n_e = int(d.sum())
        local = torch.repeat_interleave(torch.arange(b - a, device=dev), d, output_size=n_e)
        # edge j of the block, in row slot i: row_ptr[rows[i]] + (j - first slot of row i in the block)
        starts = torch.repeat_interleave(row_ptr[rows] - (torch.cumsum(d, 0) - d), d, output_size=n_e)
        out.append((rows, local, starts + torch.arange(n_e, device=dev)))
    return out


class E2AttentionArbOrder_sparse(nn.Module):
    def __init__(self, irreps_node_input="256x0e+256x1e+256x2e", attn_weight_input_dim: int = 32,
                 num_attn_heads: int = 8, attn_scalar_head: int = 32, irreps_head="32x0e+32x1e+32x2e",
                 alpha_drop=0.1, tp_type="QK_alpha", attn_type="first-order", atom_type_cnt=256,
                 norm_layer="identity", **kwargs):
        super().__init__()
        base_tp = tp_type.split("+")[0]
        if base_tp != "QK_alpha" or "softplus" in tp_type or "sigmoid" in tp_type:
            raise NotImplementedError(f"tp_type={tp_type!r}: only the default QK_alpha attention is built")
        if attn_type not in ("first-order", "so2-first-order"):
            raise NotImplementedError(f"attn_type={attn_type!r}: only the first-order SO(2) attention is built")
        self.tp_type = base_tp
        self.attn_type = attn_type
        self.atom_type_cnt = atom_type_cnt
        C, lmax = irreps_channels_lmax(irreps_node_input)
        if lmax != 2 or any(m != C for m, _, _ in parse_irreps(irreps_node_input)):
            raise NotImplementedError("node irreps must be Cx0e+Cx1e+Cx2e")
        self.scalar_dim = C
        self.lmax = lmax
        self.num_attn_heads = num_attn_heads
        self.attn_scalar_head = attn_scalar_head
        self.attn_weight_input_dim = attn_weight_input_dim
        head_mul = parse_irreps(irreps_head)[0][0]
        self.node_embed_dim = 128
        self.alpha_drop = alpha_drop
        self.source_embedding = nn.Embedding(atom_type_cnt, self.node_embed_dim)
        self.target_embedding = nn.Embedding(atom_type_cnt, self.node_embed_dim)
        nn.init.uniform_(self.source_embedding.weight.data, -0.001, 0.001)
        nn.init.uniform_(self.target_embedding.weight.data, -0.001, 0.001)
        self.edge_channel_list = [attn_weight_input_dim + self.node_embed_dim * 2,
                                  min(128, attn_weight_input_dim // 2), min(128, attn_weight_input_dim // 2)]
        self.fc_easy = RadialProfile(self.edge_channel_list + [2 * num_attn_heads])
        self.query_linear = SO3_Linear2Scalar_e2former(C, num_attn_heads * attn_scalar_head, lmax=lmax)
        self.key_linear = SO3_Linear2Scalar_e2former(C, num_attn_heads * attn_scalar_head, lmax=lmax)
        self.proj_value = SO3_Linear_e2former(C, C, lmax=lmax)
        self.first_order_tp = E2TensorProductSO2_FirstOrder(C, head_mul * num_attn_heads, lmax, num_attn_heads)
        self.proj_first = SO3_Linear_e2former(num_attn_heads * head_mul, C, lmax=lmax)
        if (29 * C) % num_attn_heads:
            raise NotImplementedError("29*C must be divisible by the number of heads")
        # keep the span's q.k scores ([E, heads] fp32) from the forward for the backward, which then
        # gathers no key rows for them (taken where the span kernels support it: 128 heads of 8)
        self.keep_logits = True
        # edge_chunk (inference path): with a number of edges set, the edge side (radial MLP and attention
        # span) runs over blocks of query rows of about that many edges, each block checkpointed: its
        # [edges, .] tensors exist only while the block runs, forward and backward (the backward forms
        # them again), so activation memory is linear in the nodes plus one block of edges
        self.edge_chunk = None

    def _fused_rows(self):
        if getattr(self, "_fused_rows_cache", None) is None:
            perm, tasks = self.first_order_tp.so2_tp.mc_row_order()
            self._fused_rows_cache = (perm, tasks)
        return self._fused_rows_cache

    def _fused_out_weights(self):
        """Per l3: proj_first.weight[l3] @ (out_linear[l3].weight * path_norm[l3]) -> [C, cnt*C'].
        The SO(2) output linear and proj_first are consecutive linear maps (no bias or activation
        between them), so one product per output row replaces the two."""
        so2 = self.first_order_tp.so2_tp
        # formed once and reused while the source tensors are unchanged (their version counters move with
        # every in-place update, e.g. an optimiser step or load_state_dict, and .to() gives them new
        # storage); this also keeps the path_norm check, a host read, out of every forward
        srcs = [self.proj_first.weight, so2.path_norm] + [so2.out_linear[i].weight
                                                           for i in range(len(so2.l3_sequential))]
        key = tuple((id(t), t._version, t.data_ptr(), t.dtype, t.device) for t in srcs)   # .to() swaps .data
        cache = getattr(self, "_fused_out_cache", None)
        if cache is not None and cache[0] == key:
            return cache[1]
        pw = self.proj_first.weight.detach()
        norm = so2.path_norm.detach().reshape(-1)
        ws = []
        for idx, (l3, cnt) in enumerate(so2.l3_sequential):
            nl = norm[l3 * l3:(l3 + 1) ** 2]
            if not bool((nl == nl[0]).all()):
                raise NotImplementedError("path_norm must be constant within an l3 block")
            ws.append(pw[l3] @ (so2.out_linear[idx].weight.detach() * nl[0]))
        self._fused_out_cache = (key, ws)
        return ws

    # -- edge radial MLP with the first layer split as W_r rbf + (W_t T)[Z_i] + (W_s S)[Z_j] + b --
    def edge_gate(self, attn_weight, atomic_numbers, f_outcell_index, query_idx, neighbor_idx):
        net = self.fc_easy.net
        lin0 = net[0]
        nb = self.attn_weight_input_dim
        e = self.node_embed_dim
        cw = not self.training
        w = lin0.weight.detach() if cw else lin0.weight
        with torch.set_grad_enabled(torch.is_grad_enabled() and not cw):
            t_tab = (self.target_embedding.weight @ w[:, nb:nb + e].t()).contiguous()   # [types, h]
            s_tab = (self.source_embedding.weight @ w[:, nb + e:].t()).contiguous()     # [types, h]
        z_q = atomic_numbers[query_idx]
        z_k = atomic_numbers[f_outcell_index][neighbor_idx]
        if isinstance(attn_weight, RbfSpec):
            h = attn_weight.linear(w[:, :nb], lin0.bias, cw)
        else:
            h = lin(attn_weight, w[:, :nb], lin0.bias, cw)
        h = run_mlp(list(net)[1:], h, cw, first_tables=(t_tab, z_q, s_tab, z_k))
        return h  # [E, 2H]: gate = [:, :H], inputhead = [:, H:]

    def _edge_chunks(self, bd, n_rows):
        """Blocks of query rows of about ``edge_chunk`` edges each, or None (the option is off, the graph
        fits one block, or its edges are not in query order).  Blocks are consecutive runs of the graph's
        spatial row order (``row_order``, else the row index), so a block's keys are a compact region.
        Per block: ``(rows, edges, md)`` = its rows in that order, its edge ids, and the CSR metadata of its
        edges with the block's rows renumbered 0..n-1.  Formed once per graph (kept in ``bd``)."""
        if not self.edge_chunk:
            return None
        rp0 = bd["metadata"][0]
        key = (self.edge_chunk, n_rows, id(rp0), rp0.data_ptr(), rp0._version)
        cached = bd.get("_edge_blocks")
        if cached is not None and cached[0] == key:
            return cached[1]
        from .ops import prepare_sparse_qk_edge_index_metadata

        row_ptr = bd["metadata"][0][: n_rows + 1].to(torch.int64)
        E = int(row_ptr[-1])
        if E <= self.edge_chunk:
            return None
        if bd.get("query_sorted", None) is None:
            qi = bd["query_idx"]
            bd["query_sorted"] = bool(qi.numel() < 2 or not bool((qi[1:] < qi[:-1]).any()))
        if not bd["query_sorted"]:
            return None
        key_sorted = bd["neighbor_idx"]
        blocks = []
        for rows, local, edges in edge_blocks(row_ptr, bd.get("row_order"), self.edge_chunk):
            md = prepare_sparse_qk_edge_index_metadata(local, key_sorted[edges], rows.numel(),
                                                       bd["f_outcell_index"].shape[0])
            blocks.append((rows, edges, md))
        bd["_edge_blocks"] = (key, blocks)
        return blocks

    def _chunk_span(self, q_scaled, key, merged, attn_weight, atomic_numbers, outcell, query_idx, neighbor_idx, poly,
                    edge_dis, rows, edges, md, key_order):
        """Radial MLP and attention span for one block of query rows (checkpointed): [rows, C', H]."""
        from torch.utils.checkpoint import checkpoint

        if isinstance(attn_weight, RbfSpec):
            aw_in, aw = attn_weight.dist[edges], attn_weight
        else:
            aw_in, aw = attn_weight[edges], None
        qi, ni = query_idx[edges], neighbor_idx[edges]

        def block(q, k, v, awd, pl, dd):
            w = RbfSpec(awd, aw.offset, aw.coeff) if aw is not None else awd
            gate = self.edge_gate(w, atomic_numbers, outcell, qi, ni)
            return attention_span(q, k, v, gate, pl, dd, md, None, key_order, keep_logits=False)

        return checkpoint(block, q_scaled[rows], key, merged, aw_in, poly[edges], edge_dis[edges],
                          use_reentrant=False)

    def forward(self, node_pos, node_irreps_input, edge_dis, edge_vec, attn_weight, atomic_numbers,
                poly_dist=None, attn_mask=None, batch=None, batched_data=None, **kwargs):
        if self.training and self.alpha_drop > 0:
            raise NotImplementedError("attention dropout (training) is not part of the inference path")
        bd = batched_data
        n_all = node_irreps_input.shape[0]
        # rows [0, N1) are queries (all rows unless the graph says otherwise: domain ghosts are keys only)
        N1 = int(bd.get("n_query", n_all))
        H = self.num_attn_heads
        C = self.scalar_dim
        outcell = bd["f_outcell_index"]
        N2 = outcell.shape[0]
        query_idx = bd["query_idx"].to(torch.long)
        neighbor_idx = bd["neighbor_idx"].to(torch.long)
        metadata = bd["metadata"]
        x = node_irreps_input

        fused = x.is_cuda and not self.training
        chunks = self._edge_chunks(bd, N1) if fused else None
        query = self.query_linear(x if N1 == n_all else x[:N1]).reshape(N1, H, -1)
        # kv_halo (domain decomposition): the rows of x are this rank's atoms only; the other atoms'
        # key / value projections come from their owners, appended after the own rows
        kv_halo = bd.get("kv_halo")
        key = self.key_linear(x)
        if kv_halo is not None:
            key = kv_halo(key, "key")
        key = key[outcell].reshape(N2, H, -1)
        q_scaled = query / math.sqrt(query.shape[-1])
        if chunks is None:
            gate = self.edge_gate(attn_weight, atomic_numbers, outcell, query_idx, neighbor_idx)

        value = self.proj_value(x)
        if kv_halo is not None:
            value = kv_halo(value, "value")
        value = value[outcell]                                                       # [N2, 9, C]
        tp = self.first_order_tp
        if fused:
            # rows of both halves in the (m, c) order of the output linear; [A_b v ; v] in one kernel
            row_perm, tasks = self._fused_rows()
            jd = bd.get("node_map_jd")
            if jd is not None:   # maps straight from positions (the caller did not form Wigner matrices)
                A_b = tp.node_map_from_pos(bd["f_exp_node_pos"], jd, row_perm)
            else:
                A_b = tp.node_map(bd["wigner_exp"], bd["wigner_inv_exp"], bd["f_exp_node_pos"], row_perm)
            merged = tc.node_apply(A_b, value, "merge")                               # [N2, 29, C]
            n_b = A_b.shape[1]
        else:
            h_b = tp.node_half(bd["wigner_exp"], bd["wigner_inv_exp"], value, bd["f_exp_node_pos"])  # [N2, 20, C]
            n_b = h_b.shape[1]
            merged = torch.cat([h_b, value], dim=1)
        merged = merged.reshape(N2, -1, H)                                              # [N2, 29*C/H, H]

        poly = poly_dist if poly_dist is not None else torch.ones_like(edge_dis)
        if chunks is not None:
            parts = [self._chunk_span(q_scaled, key, merged, attn_weight, atomic_numbers, outcell, query_idx,
                                      neighbor_idx, poly, edge_dis, rows, edges, md, bd.get("key_order"))
                     for rows, edges, md in chunks]
            rows_all = torch.cat([rows for rows, _, _ in chunks])
            agg = torch.cat(parts, dim=0)[torch.argsort(rows_all)]
        elif bd.get("query_sorted", None) is None:
            qi = bd["query_idx"]
            bd["query_sorted"] = bool(qi.numel() < 2 or not bool((qi[1:] < qi[:-1]).any()))
        if chunks is not None:
            pass
        elif bd["query_sorted"]:
            agg = attention_span(q_scaled, key, merged, gate, poly, edge_dis, metadata, bd.get("row_order"),
                                 bd.get("key_order"), keep_logits=self.keep_logits)
        else:
            # permute the edges into query-CSR order (q_perm) so that edge id == CSR slot
            perm = metadata[2].to(torch.long)
            md = (metadata[0], metadata[1], torch.arange(perm.numel(), device=perm.device, dtype=torch.int32),
                  metadata[3], metadata[4], torch.argsort(perm)[metadata[5].to(torch.long)].to(torch.int32))
            agg = attention_span(q_scaled, key, merged, gate[perm], poly[perm], edge_dis[perm], md,
                                 bd.get("row_order"), bd.get("key_order"), keep_logits=self.keep_logits)
        agg = agg.reshape(N1, -1, C)
        if fused:
            # A_a agg_v - agg_b, then output linear and proj_first as one GEMM per output row
            if jd is not None:
                A_a = tp.node_map_from_pos(node_pos[:N1], jd, row_perm)
            else:
                A_a = tp.node_map(bd["wigner"][:N1], bd["wigner_inv"][:N1], node_pos[:N1], row_perm)
            diff = tc.node_apply(A_a, agg, "sub")                                          # [N1, 20, C]
            out = tc.rowblock_linear(diff, tasks, self._fused_out_weights(), self.proj_first.bias,
                                     (self.lmax + 1) ** 2)
            return out, attn_weight
        h_b_agg, h_a = agg[:, :n_b], agg[:, n_b:]
        h_a = tp.node_half(bd["wigner"][:N1], bd["wigner_inv"][:N1], h_a, node_pos[:N1])
        out = tp.so2_tp.forward_linear(h_a - h_b_agg)
        return self.proj_first(out), attn_weight
