"""Node-side building blocks of the E2Former-V2 attention layer, with the reference's parameter
names and shapes so that reference ``state_dict``s load unchanged.

These are dense per-node contractions ([N, (lmax+1)^2, C] x [C, C']); on the GPU they run on the
tcgen05 tensor cores with the 3xTF32 split (:mod:`.linear`).  The sparse edge work lives in :mod:`.ops`.
On the CPU (used only to build / inspect modules) they fall back to plain torch arithmetic.
"""
from __future__ import annotations

import math

import torch
from torch import nn

from . import linear as tc
from .cg import so2_first_order_tables


def _degree_of_rows(lmax):
    return [l for l in range(lmax + 1) for _ in range(2 * l + 1)]


def lin(x, w, b=None, const_weights=False):
    """``F.linear`` on the tensor cores for CUDA inputs.  ``const_weights`` (eval mode) treats the
    parameters as constants, so the backward forms only the input gradient -- the one force
    evaluation needs -- instead of weight gradients nobody asked for."""
    if const_weights:
        w = w.detach()
        b = None if b is None else b.detach()
    return tc.linear(x, w, b) if x.is_cuda else nn.functional.linear(x, w, b)


def _cw(module, t):
    """Parameter as seen by the forward: a constant in eval mode."""
    return t if module.training else t.detach()


def parse_irreps(irreps):
    """Parse ``"256x0e+256x1e+256x2e"`` into ``[(mul, l, parity), ...]``."""
    if not isinstance(irreps, str):
        return [(int(m), int(ir[0]), int(ir[1]) if len(ir) > 1 else 1) for m, ir in irreps]
    out = []
    for part in irreps.split("+"):
        part = part.strip()
        if not part:
            continue
        mul, ir = part.split("x") if "x" in part else ("1", part)
        out.append((int(mul), int(ir[:-1]), 1 if ir[-1] == "e" else -1))
    return out


def irreps_channels_lmax(irreps):
    """(channels of the l=0 block, lmax) of an irreps spec with one block per l."""
    ir = parse_irreps(irreps)
    return ir[0][0], ir[-1][1]


class SO3_Linear_e2former(nn.Module):
    """Per-degree linear map ``out[:, m, :] = x[:, m, :] @ W[l(m)].T`` (+ bias on the l=0 row).

    Follows module_utils.py:2010-2055 (weight [(lmax+1), out, in], bias [out])."""

    def __init__(self, in_features, out_features, lmax, bias=True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.lmax = lmax
        self.weight = nn.Parameter(torch.empty(lmax + 1, out_features, in_features))
        bound = 1 / math.sqrt(in_features)
        nn.init.uniform_(self.weight, -bound, bound)
        self.bias = nn.Parameter(torch.zeros(out_features))
        expand_index = torch.zeros((lmax + 1) ** 2, dtype=torch.long)
        for l in range(lmax + 1):
            expand_index[l * l:(l + 1) ** 2] = l
        self.register_buffer("expand_index", expand_index, persistent=False)

    def forward(self, x):
        shape = x.shape[:-2]
        x = x.reshape(-1, x.shape[-2], x.shape[-1])
        if x.is_cuda:
            out = tc.so3_linear(x, _cw(self, self.weight), _cw(self, self.bias), _degree_of_rows(self.lmax)[: x.shape[1]])
            return out.reshape(*shape, out.shape[-2], self.out_features)
        outs = []
        for l in range(self.lmax + 1):
            blk = x[:, l * l:(l + 1) ** 2, :]
            o = torch.matmul(blk, self.weight[l].t())
            if l == 0:
                o = o + self.bias
            outs.append(o)
        out = torch.cat(outs, dim=1)
        return out.reshape(*shape, out.shape[-2], self.out_features)


class SO3_Linear2Scalar_e2former(nn.Module):
    """Two per-degree linears, per-degree inner product over m, then an MLP (module_utils.py:2198-2274)."""

    def __init__(self, in_features, out_features, lmax, hidden_features=None, bias=True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.lmax = lmax
        hidden = out_features // 2 if hidden_features is None else hidden_features
        self.hidden = hidden
        bound = 1 / math.sqrt(in_features)
        self.weight = nn.Parameter(torch.empty(lmax + 1, hidden, in_features).uniform_(-bound, bound))
        self.bias = nn.Parameter(torch.zeros(1, 1, hidden))
        self.weight2 = nn.Parameter(torch.empty(lmax + 1, hidden, in_features).uniform_(-bound, bound))
        expand_index = torch.zeros((lmax + 1) ** 2, dtype=torch.long)
        for l in range(lmax + 1):
            expand_index[l * l:(l + 1) ** 2] = l
        self.register_buffer("expand_index", expand_index)
        self.final_linear = nn.Sequential(
            nn.Linear(hidden * (lmax + 1), hidden), nn.LayerNorm(hidden), nn.SiLU(), nn.Linear(hidden, out_features))
        # inference memory mode: form the per-degree projections again in the backward instead of
        # keeping them (4 x hidden floats per irreps row)
        self.recompute_pair_product = False

    def forward(self, x):
        shape = x.shape[:-2]
        x = x.reshape(-1, x.shape[-2], x.shape[-1])
        if x.is_cuda and not self.training:
            # both projections and the inner product over m in one tensor-core GEMM per row
            h = tc.so3_pair_product(x, self.weight.detach(), self.weight2.detach(), self.bias.detach(),
                                    _degree_of_rows(self.lmax)[: x.shape[1]], recompute=self.recompute_pair_product)
            h = h.reshape(x.shape[0], -1)
            fl = self.final_linear
            cwt = not self.training
            h = lin(h, fl[0].weight, fl[0].bias, cwt)
            h = tc.ln_silu(h, fl[1]) if (cwt and tc.ln_silu_supported(h.shape[-1])) else fl[2](fl[1](h))
            h = lin(h, fl[3].weight, fl[3].bias, cwt)
            return h.reshape(*shape, self.out_features)
        # both projections in one GEMM per degree: [*, 2l+1, in] @ [in, 2*hidden]
        parts = []
        for l in range(self.lmax + 1):
            blk = x[:, l * l:(l + 1) ** 2, :]
            w = torch.cat([self.weight[l], self.weight2[l]], dim=0)
            o = torch.matmul(blk, w.t())
            o1, o2 = o[..., :self.hidden], o[..., self.hidden:]
            if l == 0:
                o1 = o1 + self.bias.reshape(1, 1, -1)
            parts.append((o1 * o2).sum(dim=1))
        out = self.final_linear(torch.cat(parts, dim=-1))
        return out.reshape(*shape, self.out_features)


class RadialProfile(nn.Module):
    """Linear -> (LayerNorm) -> SiLU ... -> Linear, parameter names as module_utils.py:2151-2178."""

    def __init__(self, ch_list, use_layer_norm=True, use_offset=True):
        super().__init__()
        mods = []
        cin = ch_list[0]
        for i in range(1, len(ch_list)):
            mods.append(nn.Linear(cin, ch_list[i], bias=use_offset))
            cin = ch_list[i]
            if i == len(ch_list) - 1:
                break
            if use_layer_norm:
                mods.append(nn.LayerNorm(ch_list[i]))
            mods.append(nn.SiLU())
        self.net = nn.Sequential(*mods)

    def forward(self, f_in):
        return run_mlp(list(self.net), f_in, not self.training)


def run_mlp(layers, h, const_weights, first_tables=None):
    """Linear / LayerNorm / SiLU stack; on CUDA in eval mode each LayerNorm+SiLU pair is one fused kernel
    (``first_tables`` are added to the first Linear's output inside that fused kernel)."""
    i = 0
    pending = first_tables
    while i < len(layers):
        layer = layers[i]
        if isinstance(layer, nn.Linear):
            h = lin(h, layer.weight, layer.bias, const_weights)
            i += 1
        elif (isinstance(layer, nn.LayerNorm) and i + 1 < len(layers) and isinstance(layers[i + 1], nn.SiLU)
              and h.is_cuda and const_weights and h.dim() == 2 and tc.ln_silu_supported(h.shape[-1])):
            h = tc.ln_silu(h, layer, pending)
            pending = None
            i += 2
            continue
        else:
            if pending is not None:
                T, zt, S, zs = pending
                h = h + T[zt] + S[zs]
                pending = None
            h = layer(h)
            i += 1
    return h


class GaussianSmearing(nn.Module):
    """``exp(coeff (d - mu_k)^2)``, mu = linspace(0, cutoff, n), coeff = -0.5 / (width*dmu)^2
    (module_utils.py:1853-1870)."""

    def __init__(self, num_basis, cutoff=5.0, basis_width_scalar=2.0):
        super().__init__()
        offset = torch.linspace(0, cutoff, num_basis)
        self.coeff = -0.5 / (basis_width_scalar * (offset[1] - offset[0])).item() ** 2
        self.register_buffer("offset", offset)

    def forward(self, dist):
        shape = dist.shape
        d = dist.view(-1, 1) - self.offset.view(1, -1)
        return torch.exp(self.coeff * torch.pow(d, 2)).reshape(*shape, -1)


class RbfSpec:
    """A Gaussian radial basis not yet formed: ``(dist [E], offsets [nb], coeff)``.  Consumers that start
    with a linear map of the basis use :func:`linear.rbf_linear`; others call :meth:`materialize`."""

    def __init__(self, dist, offset, coeff):
        self.dist, self.offset, self.coeff = dist, offset, coeff

    def materialize(self):
        d = self.dist.view(-1, 1) - self.offset.view(1, -1)
        return torch.exp(self.coeff * torch.pow(d, 2))

    def linear(self, w, b, const_weights):
        if self.dist.is_cuda and const_weights:
            return tc.rbf_linear(self.dist, self.offset, self.coeff, w, b)
        return lin(self.materialize(), w, b, const_weights)


def polynomial(dist, cutoff, exponent=5):
    """Smooth envelope 1 + r^p (a + r (b + c r)), zero for r >= 1 (module_utils.py:1946-1954)."""
    a = -(exponent + 1) * (exponent + 2) / 2
    b = exponent * (exponent + 2)
    c = -exponent * (exponent + 1) / 2
    ratio = dist / cutoff
    env = 1 + ratio ** exponent * (a + ratio * (b + c * ratio))
    return torch.where(ratio < 1, env, 0)


class SO2_TP_givenl2(nn.Module):
    """First-order (l2 = 1) SO(2) tensor product in the node frame + per-l3 output linear.

    ``forward`` selects one input row per output row and scales it by its CG coefficient
    (so2_tensor_product.py:263-271); ``forward_linear`` mixes the ``count`` paths of each l3 with
    one Linear(count*C -> C') and multiplies by 1/sqrt(count) (so2_tensor_product.py:273-290)."""

    def __init__(self, lmax=2, in_c=None, out_c=None, with_linear=True):
        super().__init__()
        _, seq, sel, w, norm = so2_first_order_tables(lmax, 1)
        self.l3_sequential = seq
        self.with_linear = with_linear
        self.in_c, self.out_c = in_c, out_c
        self.out_linear = nn.ModuleList()
        if with_linear:
            for l3, cnt in seq:
                self.out_linear.append(nn.Linear(cnt * in_c, out_c, bias=False))
        self.path_norm = nn.Parameter(torch.tensor(norm, dtype=torch.float32).reshape(1, -1, 1), requires_grad=False)
        self.selected_idx = nn.Parameter(torch.tensor(sel, dtype=torch.long), requires_grad=False)
        self.CG_weight = nn.Parameter(torch.tensor(w, dtype=torch.float32), requires_grad=False)

    def forward(self, x, with_linear=True):
        y = x[:, self.selected_idx] * self.CG_weight.reshape(1, -1, 1)
        if with_linear and self.with_linear:
            return self.forward_linear(y)
        return y

    def mc_row_order(self):
        """Row permutation (new -> old) that stores each l3 block m-major, (m, c) instead of (c, m), so
        that the ``cnt`` rows feeding output row m of an l3 block are contiguous, and the row-block
        tasks (first row, rows, output row, l3 index) of the output linear in that order."""
        perm, tasks = [], []
        start = 0
        for idx, (l3, cnt) in enumerate(self.l3_sequential):
            d = 2 * l3 + 1
            for m in range(d):
                tasks.append((start + m * cnt, cnt, l3 * l3 + m, idx))
                for c in range(cnt):
                    perm.append(start + c * d + m)
            start += d * cnt
        return perm, tasks

    def forward_linear(self, y):
        bs = y.shape[0]
        start = 0
        outs = []
        for idx, (l3, cnt) in enumerate(self.l3_sequential):
            end = start + (2 * l3 + 1) * cnt
            blk = y[:, start:end].reshape(bs, cnt, 2 * l3 + 1, -1).permute(0, 2, 1, 3).reshape(bs, 2 * l3 + 1, -1)
            outs.append(lin(blk, self.out_linear[idx].weight, None, not self.training))
            start = end
        return torch.cat(outs, dim=1) * self.path_norm


class E2TensorProductSO2_FirstOrder(nn.Module):
    """Holds the SO(2) product of the node-decomposed first-order TP (so2_tensor_product.py:293-389).
    The sparse aggregation between the two node-local halves is done by the fused attention kernel
    (see :class:`ubio_molfm_b200.attention.E2AttentionArbOrder_sparse`)."""

    def __init__(self, in_c, out_c, lmax, head):
        super().__init__()
        self.in_c, self.out_c, self.lmax, self.head = in_c, out_c, lmax, head
        self.so2_tp = SO2_TP_givenl2(lmax, in_c, out_c, with_linear=True)

    def node_map(self, wigner, wigner_inv, pos, row_perm=None):
        """A = W_inv diag(CG |pos|) S W per node, [n, 20, 9] (rows optionally permuted)."""
        tp = self.so2_tp
        scale = tp.CG_weight.reshape(1, -1, 1) * torch.norm(pos, dim=-1).reshape(-1, 1, 1)
        A = torch.bmm(wigner_inv, wigner[:, tp.selected_idx, :] * scale)
        return A if row_perm is None else A[:, row_perm]

    def node_map_from_pos(self, pos, jd, row_perm=None):
        """The same maps as :meth:`node_map`, formed by one kernel from the positions (``jd``: the
        J matrices of degrees 0..2); the Wigner matrices are never materialised."""
        # the tables are rebuilt when any source changes: the J matrices, and the selection table and CG
        # weights (state-dict entries: load_state_dict / .to() move their version counter or storage)
        tp = self.so2_tp
        srcs = [jd[1], jd[2], tp.selected_idx, tp.CG_weight]
        key = (tuple((id(t), t._version, t.data_ptr(), t.dtype, t.device) for t in srcs),
               None if row_perm is None else tuple(row_perm))
        cache = getattr(self, "_map_tables", None)
        if cache is None or cache[0] != key:
            tp = self.so2_tp
            self._map_tables = (key, tc.NodeMapTables(jd, tp.selected_idx, tp.CG_weight, row_perm))
        return tc.node_map_from_pos(pos, self._map_tables[1])

    def node_half(self, wigner, wigner_inv, h, pos):
        """W_inv @ (CG-select(W @ h) * |pos|): the per-node half of h (x) r.

        On CUDA the whole map is one per-node [20 x 9] matrix A = W_inv diag(CG |pos|) S W, built with
        small batched products (autograd carries the Wigner / position gradients) and applied to the
        [9, C] rows by one kernel."""
        tp = self.so2_tp
        if h.is_cuda:
            return tc.node_apply(self.node_map(wigner, wigner_inv, pos), h)
        y = tp(torch.bmm(wigner, h), with_linear=False) * torch.norm(pos, dim=-1).reshape(-1, 1, 1)
        return torch.bmm(wigner_inv, y)
