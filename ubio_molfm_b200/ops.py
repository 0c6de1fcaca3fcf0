"""PyTorch-facing wrappers of the C ABI: CSR metadata, the reference's kernel-level sparse ops
(same names, arguments and error behaviour as its ``triton_dr`` functions) and the fused attention
span used by :class:`ubio_molfm_b200.attention.E2AttentionArbOrder_sparse`.

Outputs are allocated through the PyTorch caching allocator and the kernels run on the current
CUDA stream.  Every op raises on non-CUDA inputs: there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, require_cuda, stream_of


class KernelTimer:
    """Optional CUDA-event bracketing of the fused-attention launches (used by the benchmark).

    Events are recorded on the current stream, the stream every kernel of this package runs on."""

    def __init__(self):
        self.enabled = False
        self.events = {}

    def start(self, name):
        if not self.enabled:
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        return (name, ev)

    def stop(self, tok):
        if tok is None:
            return
        name, s = tok
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.events.setdefault(name, []).append((s, e))

    def summary(self):
        """name -> (launches, total ms); call after synchronising."""
        return {k: (len(v), sum(s.elapsed_time(e) for s, e in v)) for k, v in self.events.items()}


TIMER = KernelTimer()


def _i32(t):
    return t.contiguous().to(torch.int32)


def _f32(t):
    return t.contiguous().to(torch.float32)


def _workspace(nbytes, device):
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


# ------------------------------------------------------------------------------------------------
# CSR metadata  (triton_sparse_qk_autograd.py:635-652)
# ------------------------------------------------------------------------------------------------
def prepare_sparse_qk_edge_index_metadata(query_index, neighbor_index, num_queries, num_keys):
    """Query-CSR and key-CSR of an edge list: ``(q_row_ptr, q_col, q_perm, k_row_ptr, k_col, k_perm)``,
    int32; the key-CSR orders the edges of a key by edge id (a stable grouping)."""
    require_cuda(query_index, neighbor_index)
    lib = _lib.load()
    dev = query_index.device
    q = _i32(query_index)
    n = _i32(neighbor_index)
    E = q.numel()
    N, M = int(num_queries), int(num_keys)
    out = [torch.empty(N + 1, dtype=torch.int32, device=dev), torch.empty(E, dtype=torch.int32, device=dev),
           torch.empty(E, dtype=torch.int32, device=dev), torch.empty(M + 1, dtype=torch.int32, device=dev),
           torch.empty(E, dtype=torch.int32, device=dev), torch.empty(E, dtype=torch.int32, device=dev)]
    ws = _workspace(lib.e2a_csr_workspace_bytes(E, N, M), dev)
    check(lib.e2a_csr_build(ptr(q), ptr(n), E, N, M, *[ptr(t) for t in out], ptr(ws), ws.numel(), stream_of(dev)),
          "e2a_csr_build (an index is out of range)")
    return tuple(out)


def _check_md(metadata):
    if metadata is None or len(metadata) != 6:
        raise ValueError("metadata must be a 6-tuple from prepare_sparse_qk_edge_index_metadata")
    return tuple(_i32(m) for m in metadata)


# ------------------------------------------------------------------------------------------------
# sparse_qk_edge_index  (triton_sparse_qk_autograd.py:839-871)
# ------------------------------------------------------------------------------------------------
def _qk_forward(query, key, md, E):
    lib = _lib.load()
    N, H, D = query.shape
    out = torch.empty((E, H), device=query.device, dtype=torch.float32)
    check(lib.e2a_sparse_qk_fwd(ptr(query), ptr(key), ptr(md[0]), ptr(md[1]), ptr(md[2]), N, E, H, D, ptr(out),
                                stream_of(query.device)), "e2a_sparse_qk_fwd")
    return out


def _grouped_reduce(alpha, x, row_ptr, col, perm, rows):
    lib = _lib.load()
    _, H, D = x.shape
    out = torch.empty((rows, H, D), device=x.device, dtype=torch.float32)
    check(lib.e2a_grouped_reduce(ptr(alpha), ptr(x), ptr(row_ptr), ptr(col), ptr(perm), rows, H, D, ptr(out),
                                 stream_of(x.device)), "e2a_grouped_reduce")
    return out


class SparseQKEdgeIndexFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, query, key, md):
        q, k = _f32(query), _f32(key)
        E = md[1].numel()
        out = _qk_forward(q, k, md, E)
        ctx.save_for_backward(query, key, *md)
        ctx.dtypes = (query.dtype, key.dtype)
        return out.to(query.dtype)

    @staticmethod
    def backward(ctx, g):
        q, k, *md = ctx.saved_tensors
        q, k = _f32(q), _f32(k)
        if torch.is_grad_enabled():
            # create_graph=True: the backward is itself a differentiable op
            # (SparseQKEdgeIndex_Fn.backward -> SparseQKEdgeBackward_Fn, triton_sparse_qk_autograd.py:725-740).
            dq, dk = SparseQKEdgeBackwardFn.apply(g, q, k, tuple(md))
            return dq.to(ctx.dtypes[0]), dk.to(ctx.dtypes[1]), None
        g = _f32(g)
        dq = dk = None
        if ctx.needs_input_grad[0]:
            dq = _grouped_reduce(g, k, md[0], md[1], md[2], q.shape[0]).to(ctx.dtypes[0])
        if ctx.needs_input_grad[1]:
            dk = _grouped_reduce(g, q, md[3], md[4], md[5], k.shape[0]).to(ctx.dtypes[1])
        return dq, dk, None


class SparseQKEdgeBackwardFn(torch.autograd.Function):
    """``(dq, dk) = backward of sparse_qk(q, k)`` at upstream gradient ``g`` as an op of its own, so that
    force-loss training can differentiate it (triton_sparse_qk_autograd.py:754-836).

    Both outputs are bilinear: ``dq = G_q(g, k)`` and ``dk = G_k(g, q)``, grouped reductions over the
    query- and key-CSR.  Their gradients therefore reuse the same two kernels:
    ``d g = qk(gg_dq, k) + qk(q, gg_dk)``, ``d q = G_q(g, gg_dk)``, ``d k = G_k(g, gg_dq)``."""

    @staticmethod
    def forward(ctx, g, q, k, md):
        g = _f32(g)
        dq = _grouped_reduce(g, k, md[0], md[1], md[2], q.shape[0])
        dk = _grouped_reduce(g, q, md[3], md[4], md[5], k.shape[0])
        ctx.save_for_backward(g, q, k, *md)
        return dq, dk

    @staticmethod
    def backward(ctx, gg_dq, gg_dk):
        g, q, k, *md = ctx.saved_tensors
        E = g.shape[0]
        d_g = d_q = d_k = None
        gg_dq = None if gg_dq is None else _f32(gg_dq)
        gg_dk = None if gg_dk is None else _f32(gg_dk)
        if ctx.needs_input_grad[0]:
            d_g = torch.zeros_like(g)
            if gg_dq is not None:
                d_g += _qk_forward(gg_dq, k, md, E)
            if gg_dk is not None:
                d_g += _qk_forward(q, gg_dk, md, E)
        if ctx.needs_input_grad[1] and gg_dk is not None:
            d_q = _grouped_reduce(g, gg_dk, md[0], md[1], md[2], q.shape[0])
        if ctx.needs_input_grad[2] and gg_dq is not None:
            d_k = _grouped_reduce(g, gg_dq, md[3], md[4], md[5], k.shape[0])
        return d_g, d_q, d_k, None


def sparse_qk_edge_index(query, key, query_index, neighbor_index, metadata=None):
    """``out[e, h] = <query[query_index[e], h], key[neighbor_index[e], h]>`` -> [E, H]."""
    require_cuda(query, key, query_index, neighbor_index)
    if query.ndim != 3 or key.ndim != 3 or query.shape[1:] != key.shape[1:]:
        raise ValueError("query must be [N,H,D] and key [M,H,D]")
    if metadata is None:
        metadata = prepare_sparse_qk_edge_index_metadata(query_index, neighbor_index, query.shape[0], key.shape[0])
    md = _check_md(metadata)
    return SparseQKEdgeIndexFn.apply(query, key, md)


# ------------------------------------------------------------------------------------------------
# sparse_alpha_sum_edge_index  (sparse_alpha_sum_edge_index_autograd.py:207-213)
# ------------------------------------------------------------------------------------------------
def prepare_sparse_alpha_sum_edge_index_metadata(query_index, num_queries):
    md = prepare_sparse_qk_edge_index_metadata(query_index, query_index, num_queries, num_queries)
    return md[0], md[2]


class SparseAlphaSumFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, alpha, query_index, row_ptr, perm, num_queries):
        a = _f32(alpha)
        out = _alpha_sum(a, row_ptr, perm, num_queries)
        ctx.save_for_backward(_i32(query_index), row_ptr, perm)
        ctx.shape = a.shape
        ctx.dtype = alpha.dtype
        return out.to(alpha.dtype)

    @staticmethod
    def backward(ctx, g):
        qi, row_ptr, perm = ctx.saved_tensors
        if torch.is_grad_enabled():
            # sparse_alpha_sum_edge_index_autograd.py:145-155 (SparseAlphaSumEdgeIndexBackwardFn)
            ga = SparseAlphaSumBackwardFn.apply(g, qi, row_ptr, perm, ctx.shape)
        else:
            ga = _alpha_gather(_f32(g), qi, ctx.shape)
        return ga.to(ctx.dtype), None, None, None, None


def _alpha_gather(g, qi, shape):
    lib = _lib.load()
    E, H = shape
    ga = torch.empty((E, H), device=g.device, dtype=torch.float32)
    check(lib.e2a_alpha_sum_bwd(ptr(g), ptr(qi), E, H, ptr(ga), stream_of(g.device)), "e2a_alpha_sum_bwd")
    return ga


def _alpha_sum(a, row_ptr, perm, num_queries):
    lib = _lib.load()
    H = a.shape[1]
    out = torch.empty((num_queries, H), device=a.device, dtype=torch.float32)
    check(lib.e2a_alpha_sum_fwd(ptr(a), ptr(row_ptr), ptr(perm), num_queries, H, ptr(out), stream_of(a.device)),
          "e2a_alpha_sum_fwd")
    return out


class SparseAlphaSumBackwardFn(torch.autograd.Function):
    """The alpha-sum backward (``ga[e] = g[query_index[e]]``, a gather) as a differentiable op; its
    gradient is the segmented sum again (sparse_alpha_sum_edge_index_autograd.py:173-208)."""

    @staticmethod
    def forward(ctx, g, qi, row_ptr, perm, shape):
        ctx.save_for_backward(row_ptr, perm)
        ctx.rows = g.shape[0]
        return _alpha_gather(_f32(g), qi, shape)

    @staticmethod
    def backward(ctx, gg):
        row_ptr, perm = ctx.saved_tensors
        d_g = _alpha_sum(_f32(gg), row_ptr, perm, ctx.rows) if ctx.needs_input_grad[0] else None
        return d_g, None, None, None, None


def sparse_alpha_sum_edge_index(alpha, query_index, num_queries, metadata=None):
    """``out[n, h] = sum_{e: query_index[e] = n} alpha[e, h]`` -> [N, H]; metadata = (row_ptr, perm)."""
    require_cuda(alpha, query_index)
    if metadata is None:
        metadata = prepare_sparse_alpha_sum_edge_index_metadata(query_index, num_queries)
    row_ptr, perm = (_i32(m) for m in metadata)
    return SparseAlphaSumFn.apply(alpha, query_index, row_ptr, perm, int(num_queries))


# ------------------------------------------------------------------------------------------------
# sparse_v_agg_edge_index_cblocked  (sparse_v_agg_edge_index_cblocked_bench.py:428-449)
# ------------------------------------------------------------------------------------------------
def _v_agg(v, a, md, num_queries):
    """``out[n, c, h] = sum_{e in row n} a[e, h] * v[key_e, c, h]`` over the query-CSR."""
    lib = _lib.load()
    M, C, H = v.shape
    out = torch.empty((num_queries, C, H), device=v.device, dtype=torch.float32)
    check(lib.e2a_v_agg_fwd(ptr(v), ptr(a), ptr(md[0]), ptr(md[1]), ptr(md[2]), num_queries, C, H, ptr(out),
                            stream_of(v.device)), "e2a_v_agg_fwd")
    return out


def _v_agg_dvalue(a, g, md, M):
    """``dv[m, c, h] = sum_{e with key m} a[e, h] * g[query_e, c, h]`` over the key-CSR."""
    lib = _lib.load()
    _, C, H = g.shape
    dv = torch.empty((M, C, H), device=g.device, dtype=torch.float32)
    check(lib.e2a_v_agg_bwd_value(ptr(a), ptr(g), ptr(md[3]), ptr(md[4]), ptr(md[5]), M, C, H, ptr(dv),
                                  stream_of(g.device)), "e2a_v_agg_bwd_value")
    return dv


def _v_agg_dalpha(g, v, md):
    """``da[e, h] = sum_c g[query_e, c, h] * v[key_e, c, h]``."""
    lib = _lib.load()
    N, C, H = g.shape
    da = torch.empty((md[1].numel(), H), device=g.device, dtype=torch.float32)
    check(lib.e2a_v_agg_bwd_alpha(ptr(g), ptr(v), ptr(md[0]), ptr(md[1]), ptr(md[2]), N, C, H, ptr(da),
                                  stream_of(g.device)), "e2a_v_agg_bwd_alpha")
    return da


def _v_agg_bf16(v, a, md, num_queries):
    """:func:`_v_agg` reading bf16 value rows directly (widened in the gather); None where the entry point
    does not take the layout."""
    lib = _lib.load()
    M, C, H = v.shape
    out = torch.empty((num_queries, C, H), device=v.device, dtype=torch.float32)
    rc = lib.e2a_v_agg_fwd_bf16(ptr(v), ptr(a), ptr(md[0]), ptr(md[1]), ptr(md[2]), num_queries, C, H, ptr(out),
                                stream_of(v.device))
    if rc == _lib.E2A_ERR_UNSUPPORTED:
        return None
    check(rc, "e2a_v_agg_fwd_bf16")
    return out


class SparseVAggFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, value, alpha, md, num_queries):
        out = None
        if value.dtype == torch.bfloat16:
            out = _v_agg_bf16(value.contiguous(), _f32(alpha), md, num_queries)
        if out is None:
            out = _v_agg(_f32(value), _f32(alpha), md, num_queries)
        ctx.save_for_backward(value, alpha, *md)
        ctx.dtypes = (value.dtype, alpha.dtype)
        return out.to(value.dtype)

    @staticmethod
    def backward(ctx, g):
        v, a, *md = ctx.saved_tensors
        v, a = _f32(v), _f32(a)
        if torch.is_grad_enabled():
            # sparse_v_agg_edge_index_cblocked_bench.py:334-347 (SparseVAggEdgeIndexCBlocked_Backward_Fn)
            dv, da = SparseVAggBackwardFn.apply(g, v, a, tuple(md))
            return dv.to(ctx.dtypes[0]), da.to(ctx.dtypes[1]), None, None
        g = _f32(g)
        dv = da = None
        if ctx.needs_input_grad[0]:
            dv = _v_agg_dvalue(a, g, md, v.shape[0]).to(ctx.dtypes[0])
        if ctx.needs_input_grad[1]:
            da = _v_agg_dalpha(g, v, md).to(ctx.dtypes[1])
        return dv, da, None, None


class SparseVAggBackwardFn(torch.autograd.Function):
    """``(dv, da)`` of the value aggregation as a differentiable op
    (sparse_v_agg_edge_index_cblocked_bench.py:361-420).  ``dv`` is bilinear in ``(a, g)`` and ``da`` in
    ``(g, v)``, so the second-order terms are the same three kernels with other operands:
    ``d g = agg(gg_dv, a) + agg(v, gg_da)``, ``d v = dvalue(gg_da, g)``, ``d a = dalpha(g, gg_dv)``."""

    @staticmethod
    def forward(ctx, g, v, a, md):
        g = _f32(g)
        dv = _v_agg_dvalue(a, g, md, v.shape[0])
        da = _v_agg_dalpha(g, v, md)
        ctx.save_for_backward(g, v, a, *md)
        return dv, da

    @staticmethod
    def backward(ctx, gg_dv, gg_da):
        g, v, a, *md = ctx.saved_tensors
        gg_dv = None if gg_dv is None else _f32(gg_dv)
        gg_da = None if gg_da is None else _f32(gg_da)
        d_g = d_v = d_a = None
        if ctx.needs_input_grad[0]:
            d_g = torch.zeros_like(g)
            if gg_dv is not None:
                d_g += _v_agg(gg_dv, a, md, g.shape[0])
            if gg_da is not None:
                d_g += _v_agg(v, gg_da, md, g.shape[0])
        if ctx.needs_input_grad[1] and gg_da is not None:
            d_v = _v_agg_dvalue(gg_da, g, md, v.shape[0])
        if ctx.needs_input_grad[2] and gg_dv is not None:
            d_a = _v_agg_dalpha(g, gg_dv, md)
        return d_g, d_v, d_a, None


def sparse_v_agg_edge_index_cblocked(value, alpha, query_index, value_index, num_queries, metadata=None):
    """``out[query_index[e], c, h] += alpha[e, h] * value[value_index[e], c, h]`` -> [N, C, H]."""
    require_cuda(value, alpha, query_index, value_index)
    if value.ndim != 3:
        raise ValueError("value must be [M, C, H]")
    if alpha.ndim != 2:
        raise ValueError("alpha must be [E, H]")
    if metadata is None:
        metadata = prepare_sparse_qk_edge_index_metadata(query_index, value_index, num_queries, value.shape[0])
    md = _check_md(metadata)
    return SparseVAggFn.apply(value, alpha, md, int(num_queries))


# ------------------------------------------------------------------------------------------------
# edge_degree_outer  (edge_degree_outer_autograd.py:348-375)
# ------------------------------------------------------------------------------------------------
def _edge_outer(sh, fea, row_ptr, perm, num_queries):
    lib = _lib.load()
    E, L = sh.shape
    F = fea.shape[1]
    out = torch.empty((num_queries, L, F), device=sh.device, dtype=torch.float32)
    check(lib.e2a_edge_outer_fwd(ptr(sh), ptr(fea), ptr(row_ptr), ptr(perm), num_queries, L, F, ptr(out),
                                 stream_of(sh.device)), "e2a_edge_outer_fwd")
    return out


def _edge_outer_bwd(g, sh, fea, qi, want_sh, want_fea):
    """``d_sh[e, l] = sum_f g[q_e, l, f] fea[e, f]`` and ``d_fea[e, f] = sum_l g[q_e, l, f] sh[e, l]``
    (either may be skipped; a skipped one's other operand is not read)."""
    lib = _lib.load()
    E, L = sh.shape
    F = g.shape[2]
    dsh = torch.empty((E, L), device=g.device, dtype=torch.float32) if want_sh else None
    dfea = torch.empty((E, F), device=g.device, dtype=torch.float32) if want_fea else None
    if dsh is not None or dfea is not None:
        check(lib.e2a_edge_outer_bwd(ptr(g), ptr(sh), ptr(fea), ptr(qi), E, L, F, ptr(dsh), ptr(dfea),
                                     stream_of(g.device)), "e2a_edge_outer_bwd")
    return dsh, dfea


class EdgeDegreeOuterFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, edge_sh, edge_fea, query_index, row_ptr, perm, num_queries):
        out = _edge_outer(_f32(edge_sh), _f32(edge_fea), row_ptr, perm, num_queries)
        ctx.save_for_backward(edge_sh, edge_fea, _i32(query_index), row_ptr, perm)
        ctx.dtypes = (edge_sh.dtype, edge_fea.dtype)
        return out.to(edge_fea.dtype)

    @staticmethod
    def backward(ctx, g):
        sh, fea, qi, row_ptr, perm = ctx.saved_tensors
        sh, fea = _f32(sh), _f32(fea)
        if torch.is_grad_enabled():
            # edge_degree_outer_autograd.py:316-325 (EdgeDegreeOuterBackward_Fn)
            dsh, dfea = EdgeDegreeOuterBackwardFn.apply(g, sh, fea, qi, row_ptr, perm)
        else:
            dsh, dfea = _edge_outer_bwd(_f32(g), sh, fea, qi, ctx.needs_input_grad[0], ctx.needs_input_grad[1])
        return (None if dsh is None else dsh.to(ctx.dtypes[0]), None if dfea is None else dfea.to(ctx.dtypes[1]),
                None, None, None, None)


class EdgeDegreeOuterBackwardFn(torch.autograd.Function):
    """``(d_sh, d_fea)`` of the edge-degree outer product as a differentiable op
    (edge_degree_outer_autograd.py:259-296): ``d g = outer(gg_dsh, fea) + outer(sh, gg_dfea)``,
    ``d sh = d_sh-kernel(g, gg_dfea)``, ``d fea = d_fea-kernel(g, gg_dsh)``."""

    @staticmethod
    def forward(ctx, g, sh, fea, qi, row_ptr, perm):
        g = _f32(g)
        dsh, dfea = _edge_outer_bwd(g, sh, fea, qi, True, True)
        ctx.save_for_backward(g, sh, fea, qi, row_ptr, perm)
        return dsh, dfea

    @staticmethod
    def backward(ctx, gg_dsh, gg_dfea):
        g, sh, fea, qi, row_ptr, perm = ctx.saved_tensors
        gg_dsh = None if gg_dsh is None else _f32(gg_dsh)
        gg_dfea = None if gg_dfea is None else _f32(gg_dfea)
        d_g = d_sh = d_fea = None
        if ctx.needs_input_grad[0]:
            d_g = torch.zeros_like(g)
            if gg_dsh is not None:
                d_g += _edge_outer(gg_dsh, fea, row_ptr, perm, g.shape[0])
            if gg_dfea is not None:
                d_g += _edge_outer(sh, gg_dfea, row_ptr, perm, g.shape[0])
        if ctx.needs_input_grad[1] and gg_dfea is not None:
            d_sh = _edge_outer_bwd(g, sh, gg_dfea, qi, True, False)[0]
        if ctx.needs_input_grad[2] and gg_dsh is not None:
            d_fea = _edge_outer_bwd(g, gg_dsh, fea, qi, False, True)[1]
        return d_g, d_sh, d_fea, None, None, None


def edge_degree_outer(edge_sh, edge_fea, query_index, num_queries, metadata=None):
    """``out[n, l, h] = sum_{e: query_index[e] = n} edge_sh[e, l] * edge_fea[e, h]`` -> [N, L, H]."""
    require_cuda(edge_sh, edge_fea, query_index)
    if metadata is None:
        md = prepare_sparse_qk_edge_index_metadata(query_index, torch.arange(query_index.numel(),
                                                                             device=query_index.device),
                                                   num_queries, query_index.numel())
    elif isinstance(metadata, (tuple, list)):
        if len(metadata) != 6:
            raise ValueError("metadata must be a 6-tuple")
        md = metadata
    else:
        raise ValueError("metadata must be a tuple/list")
    return EdgeDegreeOuterFn.apply(edge_sh, edge_fea, query_index, _i32(md[0]), _i32(md[2]), int(num_queries))


# Names of the reference's kernel API (the "triton" suffix is kept so callers need no edit).
sparse_qk_edge_index_triton = sparse_qk_edge_index
sparse_alpha_sum_edge_index_triton = sparse_alpha_sum_edge_index
sparse_v_agg_edge_index_triton_cblocked = sparse_v_agg_edge_index_cblocked
edge_degree_outer_triton = edge_degree_outer


# ------------------------------------------------------------------------------------------------
# Fused attention span
# ------------------------------------------------------------------------------------------------
class AttnSpanFn(torch.autograd.Function):
    """QK logits -> gated segmented softmax -> alpha/r -> value aggregation, and its backward.

    Inputs (fp32, CUDA): q_scaled [N,H,D], key [M,H,D], value [M,C,H], edge_gate [E,2H] (gate =
    [:, :H], inputhead = [:, H:]), poly [E], dist [E], and the CSR of the (query-sorted) edge list.
    """

    @staticmethod
    def forward(ctx, q, key, value, edge_gate, poly, dist, md, row_order, key_order, keep_logits=False):
        lib = _lib.load()
        q_in, key_in, value_in, edge_gate_in, poly_in, dist_in = q, key, value, edge_gate, poly, dist
        q, key, value = _f32(q), _f32(key), _f32(value)
        edge_gate, poly, dist = _f32(edge_gate), _f32(poly), _f32(dist)
        N, H, D = q.shape
        M, C, H2 = value.shape
        E = edge_gate.shape[0]
        if H2 != H or edge_gate.shape[1] != 2 * H or key.shape != (M, H, D):
            raise ValueError("inconsistent attention span shapes")
        dev = q.device
        out = torch.empty((N, C, H), device=dev, dtype=torch.float32)
        beta = torch.empty((E, H), device=dev, dtype=torch.float32)
        rmax = torch.empty((N, H), device=dev, dtype=torch.float32)
        rsum = torch.empty((N, H), device=dev, dtype=torch.float32)
        # the q.k scores are kept only where the backward's fused key-side path and the warp layout run
        keep = bool(keep_logits) and span_keeps_logits(H, D) and any(ctx.needs_input_grad[:6])
        logits = torch.empty((E, H), device=dev, dtype=torch.float32) if keep else None
        tok = TIMER.start("e2a_attn_fwd")
        check(lib.e2a_attn_fwd_logits(ptr(q), ptr(key), ptr(value), ptr(edge_gate), ptr(edge_gate[:, H:]), 2 * H,
                                      ptr(poly), ptr(dist), ptr(md[0]), ptr(md[1]), ptr(row_order), N, M, E, H, D,
                                      C, ptr(out), ptr(beta), ptr(rmax), ptr(rsum), ptr(logits), stream_of(dev)),
              "e2a_attn_fwd")
        TIMER.stop(tok)
        # the caller's own tensors too (the same objects, no copies, where they are already fp32 and
        # contiguous): a create_graph backward differentiates through them
        ctx.save_for_backward(q, key, value, edge_gate, poly, dist, beta, rmax, rsum, logits, row_order, key_order,
                              q_in, key_in, value_in, edge_gate_in, poly_in, dist_in, *md)
        return out

    @staticmethod
    def backward(ctx, dout):
        (q, key, value, edge_gate, poly, dist, beta, rmax, rsum, logits, row_order, key_order,
         *rest) = ctx.saved_tensors
        inputs, md = tuple(rest[:6]), rest[6:]
        if torch.is_grad_enabled():
            return _span_double_backward(ctx, inputs, dout, md)
        lib = _lib.load()
        dout = _f32(dout)
        N, H, D = q.shape
        M, C, _ = value.shape
        E = edge_gate.shape[0]
        dev = q.device
        st = stream_of(dev)
        d_q = torch.empty_like(q)
        d_gate = torch.empty((E, 2 * H), device=dev, dtype=torch.float32)
        d_poly = torch.empty(E, device=dev, dtype=torch.float32)
        d_dist = torch.empty(E, device=dev, dtype=torch.float32)
        d_logit = torch.empty((E, H), device=dev, dtype=torch.float32)
        d_k = torch.empty_like(key)
        d_v = torch.empty_like(value)
        if H <= 128 and 1024 % H == 0:
            # fused key-side pass first (d_value and d_beta from one gather of each cotangent row)
            d_beta = torch.empty((E, H), device=dev, dtype=torch.float32)
            tok = TIMER.start("e2a_attn_bwd_value")
            check(lib.e2a_attn_bwd_value(ptr(value), ptr(dout), ptr(beta), ptr(md[3]), ptr(md[4]), ptr(md[5]),
                                         ptr(key_order), N, M, E, H, D, C, ptr(d_v), ptr(d_beta), st),
                  "e2a_attn_bwd_value")
            TIMER.stop(tok)
            tok = TIMER.start("e2a_attn_bwd_softmax")
            if logits is not None:
                check(lib.e2a_attn_bwd_softmax_logits(
                    ptr(key), ptr(edge_gate), ptr(edge_gate[:, H:]), 2 * H, ptr(poly), ptr(dist), ptr(md[0]),
                    ptr(md[1]), ptr(row_order), N, M, E, H, D, C, ptr(beta), ptr(rmax), ptr(rsum), ptr(logits),
                    ptr(d_beta), ptr(d_q), ptr(d_gate), ptr(d_gate[:, H:]), 2 * H, ptr(d_poly), ptr(d_dist),
                    ptr(d_logit), st), "e2a_attn_bwd_softmax_logits")
            else:
                ws = _workspace(lib.e2a_attn_bwd_softmax_workspace_bytes(E, H), dev)
                check(lib.e2a_attn_bwd_softmax(ptr(q), ptr(key), ptr(edge_gate), ptr(edge_gate[:, H:]), 2 * H,
                                               ptr(poly), ptr(dist), ptr(md[0]), ptr(md[1]), ptr(row_order), N, M, E,
                                               H, D, C,
                                               ptr(beta), ptr(rmax), ptr(rsum), ptr(d_beta), ptr(d_q), ptr(d_gate),
                                               ptr(d_gate[:, H:]), 2 * H, ptr(d_poly), ptr(d_dist), ptr(d_logit),
                                               ptr(ws), ws.numel(), st), "e2a_attn_bwd_softmax")
            TIMER.stop(tok)
            tok = TIMER.start("e2a_attn_bwd_dk")
            check(lib.e2a_attn_bwd_dk(ptr(q), ptr(d_logit), ptr(md[3]), ptr(md[4]), ptr(md[5]), ptr(key_order), N, M,
                                      E, H, D, C, ptr(d_k), st), "e2a_attn_bwd_dk")
            TIMER.stop(tok)
            return d_q, d_k, d_v, d_gate, d_poly, d_dist, None, None, None, None
        ws = _workspace(lib.e2a_attn_bwd_workspace_bytes(E, H), dev)
        tok = TIMER.start("e2a_attn_bwd_query")
        check(lib.e2a_attn_bwd_query(ptr(q), ptr(key), ptr(value), ptr(edge_gate), ptr(edge_gate[:, H:]), 2 * H,
                                     ptr(poly), ptr(dist), ptr(md[0]), ptr(md[1]), ptr(row_order), N, M, E, H, D, C,
                                     ptr(beta), ptr(rmax), ptr(rsum), ptr(dout), ptr(d_q), ptr(d_gate),
                                     ptr(d_gate[:, H:]), 2 * H, ptr(d_poly), ptr(d_dist), ptr(d_logit), ptr(ws),
                                     ws.numel(), st), "e2a_attn_bwd_query")
        TIMER.stop(tok)
        tok = TIMER.start("e2a_attn_bwd_key")
        check(lib.e2a_attn_bwd_key(ptr(q), ptr(dout), ptr(beta), ptr(d_logit), ptr(md[3]), ptr(md[4]), ptr(md[5]),
                                   ptr(key_order), N, M, E, H, D, C, ptr(d_k), ptr(d_v), st), "e2a_attn_bwd_key")
        TIMER.stop(tok)
        return d_q, d_k, d_v, d_gate, d_poly, d_dist, None, None, None, None


def _span_composite(q, key, value, edge_gate, poly, dist, md, N):
    """The span as a chain of differentiable ops -- the kernel-level q.k and value-aggregation ops (each with
    its own double backward) around the gated segmented softmax in PyTorch elementwise / scatter ops,
    written as the reference writes it (e2former.py:311-364, 422), including its ``amax`` reduction."""
    H = q.shape[1]
    rows = torch.repeat_interleave(torch.arange(N, device=q.device), (md[0][1:] - md[0][:-1]).long())
    qi = torch.empty_like(rows)
    qi[md[2].long()] = rows                                   # query row of each edge id
    gate, inputhead = edge_gate[:, :H], edge_gate[:, H:]
    alpha = gate * SparseQKEdgeIndexFn.apply(q, key, md)
    idx = qi.unsqueeze(-1).expand(-1, H)
    amax = torch.full((N, H), -torch.inf, device=q.device, dtype=alpha.dtype)
    amax = amax.scatter_reduce(0, idx, alpha, reduce="amax", include_self=True)
    alpha = torch.exp(alpha - amax[qi]) * poly.unsqueeze(-1)
    asum = torch.zeros((N, H), device=q.device, dtype=alpha.dtype).scatter_add(0, idx, alpha)
    alpha = alpha * inputhead / (asum[qi] + 1e-3)
    alpha = alpha / dist.unsqueeze(-1).clamp_min(1e-6)
    return SparseVAggFn.apply(value, alpha, md, N)


def _span_double_backward(ctx, ins, dout, md):
    """Backward of :class:`AttnSpanFn` under ``create_graph=True`` (force-loss training): the span is formed
    again from :func:`_span_composite` and differentiated with a graph, so the returned gradients are
    themselves differentiable in the inputs and in ``dout``.  The first-order values equal the fused
    kernels' up to fp32 rounding; the fused kernels keep serving every first-order backward."""
    need = [bool(n) for n in ctx.needs_input_grad[:6]]
    with torch.enable_grad():
        # one fresh view per input: the inputs may depend on one another (poly and the radial gate are
        # functions of dist), and a gradient w.r.t. the tensors themselves would be the total derivative
        f32 = [t.contiguous().to(torch.float32).view_as(t) for t in ins]
        out = _span_composite(*f32, tuple(md), int(ins[0].shape[0]))
        wrt = [t for t, n in zip(f32, need) if n]
        got = iter(torch.autograd.grad(out, wrt, dout, create_graph=True, allow_unused=True))
    grads = [next(got) if n else None for n in need]
    grads = [None if g is None else g.to(t.dtype) for g, t in zip(grads, ins)]
    return (*grads, None, None, None, None)


def span_keeps_logits(H, D):
    """Whether :class:`AttnSpanFn` can keep the q.k scores for its backward at this head layout
    (128 heads of 8: the warp-per-row softmax kernels, with the fused key-side backward)."""
    return H == 128 and D == 8


def attention_span(q_scaled, key, value, edge_gate, poly, dist, metadata, row_order=None, key_order=None,
                   keep_logits=False):
    """Fused attention span (see :class:`AttnSpanFn`); ``metadata`` is the 6-tuple CSR of a
    query-sorted edge list (identity query permutation).  ``keep_logits``: keep the q.k scores
    ([E, H] fp32) for the backward instead of recomputing them from gathered key rows (taken where
    :func:`span_keeps_logits`; the gradients are the same bit for bit)."""
    require_cuda(q_scaled, key, value, edge_gate, poly, dist)
    md = _check_md(metadata)
    ro = None if row_order is None else _i32(row_order)
    ko = None if key_order is None else _i32(key_order)
    return AttnSpanFn.apply(q_scaled, key, value, edge_gate, poly, dist, md, ro, ko, bool(keep_logits))
