"""Radius-graph construction on the GPU behind the reference's call signatures.

* :func:`pbc_image_offsets` -- the image cells ``CellExpander`` considers (module_utils.py:871-1001),
  computed on the host with the same fp32 torch operations.
* :func:`expand_pbc` -- ``CellExpander.expand_includeself`` (module_utils.py:1065-1275) for one
  periodic system: cell-list existence test per image on the GPU.
* :func:`distributed_cell_expand` -- the image expansion of the reference's FAISS neighbour path
  (sp/dist_ner.py:27-84): its expanded-node order (candidate cells in i-j-k order, atoms ascending,
  kept by their box distance to the atoms' bounding box).
* :func:`radius_graph` -- the flattened (pyG-style) radius graph: cell-list neighbour search,
  (distance, index)-ordered rows, ``max_neighbors`` truncation, CSR metadata and a spatial row order.
* :func:`construct_radius_neighbor` -- the reference's padded ``[B, L]`` API (module_utils.py:3119).

Edge sets and distances are bit-exact with the reference (same fp32 operation sequence for every
distance).  Within a row the reference orders neighbours with an unstable sort; rows whose distances
are all distinct therefore match it exactly, and exact ties are ordered here by expanded-node index.
Edge vectors and distances are returned as differentiable functions of the positions.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, require_cuda, stream_of
from .nn import polynomial
from .ops import prepare_sparse_qk_edge_index_metadata


def _ws(nbytes, device):
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


# ------------------------------------------------------------------------------------------------
# PBC image expansion
# ------------------------------------------------------------------------------------------------
def _candidate_cells(n):
    cells = [[i, j, k] for i in range(-n, n + 1) for j in range(-n, n + 1) for k in range(-n, n + 1)
             if not (i == 0 and j == 0 and k == 0)]
    return torch.tensor(cells)


def pbc_image_offsets(cell, pbc, cutoff, num_cell_per_direction=4):
    """Image translations kept for one system, in the reference's order (home cell first).

    ``cell`` [3,3] (rows are lattice vectors), ``pbc`` [3] bool.  The per-direction reach
    ``ceil(cutoff / |n_d . a_d|)`` and the fp32 ``offset = n @ cell`` follow module_utils.py:956-999 and
    1092-1104; cells with a non-zero shift along a non-periodic direction are dropped as in 1151-1157.
    """
    return pbc_image_cells(cell, pbc, cutoff, num_cell_per_direction)[1]


def pbc_image_cells(cell, pbc, cutoff, num_cell_per_direction=4):
    """``(cells [K,3] int64, offsets [K,3] fp32)``: the integer cell shifts n of
    :func:`pbc_image_offsets` (same order) with their translations ``n @ cell``."""
    cell = torch.as_tensor(cell, dtype=torch.float32).reshape(1, 3, 3).cpu()
    pbc = torch.as_tensor(pbc, dtype=torch.bool).reshape(3).cpu()
    cells = _candidate_cells(num_cell_per_direction)
    max_off = []
    for d in range(3):
        try:
            a0 = cell[:, d, :]
            a12 = cell[:, torch.arange(3) != d, :]
            nv = torch.cross(a12[:, 0, :], a12[:, 1, :], dim=-1)
            nv = nv / nv.norm(dim=-1, keepdim=True)
            mo = int(torch.max(torch.ceil(cutoff / torch.abs(torch.sum(nv * a0, dim=-1)))))
        except Exception:
            mo = num_cell_per_direction
        max_off.append(mo)
    mask = (cells.abs() <= torch.tensor(max_off)).all(dim=-1)
    sel = cells[mask]
    sel = torch.cat([torch.zeros((1, 3), dtype=sel.dtype), sel], dim=0)
    allowed = torch.all(pbc.unsqueeze(0) >= (sel != 0), dim=-1)
    sel = sel[allowed]
    offsets = torch.bmm(sel.to(torch.float32).unsqueeze(0), cell)[0]
    return sel.to(torch.int64), offsets.contiguous()


def expand_pbc(pos, cell, pbc, cutoff, num_cell_per_direction=4):
    """Periodic images of one system within ``cutoff`` of any atom.

    Returns ``(exp_pos [N2,3], outcell [N2] int64, image [N2] int64)`` with the home cell first, then
    the kept images in the reference's cell order, atoms ascending.  ``exp_pos`` is differentiable in
    ``pos`` (``pos[outcell] + offset[image]``, the same fp32 addition as the reference)."""
    require_cuda(pos)
    lib = _lib.load()
    dev = pos.device
    offsets = pbc_image_offsets(cell, pbc, cutoff, num_cell_per_direction).to(dev)
    n_img = offsets.shape[0]
    n = pos.shape[0]
    p32 = pos.detach().to(torch.float32).contiguous()
    exp_buf = torch.empty((n_img * n, 3), dtype=torch.float32, device=dev)
    img_atom = torch.empty(n_img * n, dtype=torch.int64, device=dev)
    n_out = torch.zeros(1, dtype=torch.int64)
    ws = _ws(lib.e2a_pbc_expand_workspace_bytes(n, n_img), dev)
    import ctypes
    cnt = ctypes.c_int64(0)
    check(lib.e2a_pbc_expand(ptr(p32), n, ptr(offsets), n_img, float(cutoff), ptr(exp_buf), ptr(img_atom),
                             ctypes.byref(cnt), ptr(ws), ws.numel(), stream_of(dev)), "e2a_pbc_expand")
    del n_out
    k = int(cnt.value)
    img_atom = img_atom[:k]
    outcell = img_atom % n
    image = img_atom // n
    exp_pos = pos.to(torch.float32)[outcell] + offsets[image]
    return exp_pos, outcell, image


def distributed_cell_expand(pos, cell_size, cutoff, cell_boundMIN, cell_boundMAX, num_cell_perdirection=1,
                            pbc=None):
    """Image expansion of the reference's FAISS neighbour path (``distributed_cell_expand``,
    sp/dist_ner.py:27-84, called from e2former_wrapper.py:179-191 with the atoms' bounding box).

    ``pos`` [1, N, 3] (one system).  The candidate cells are i, j, k in [-n, n] (only 0 along a
    non-periodic direction), i slowest; every cell contributes all atoms in order, translated by
    ``[i, j, k] @ cell_size``; an image is kept when its distance to the box [``cell_boundMIN``,
    ``cell_boundMAX``] is below ``cutoff``.  The home cell is not first (it sits in the middle of the
    candidate order), unlike ``CellExpander``.  Same fp32 operations as the reference, so the kept
    set and the positions are bit-identical on the same device; differentiable in ``pos``.  Returns the
    reference's dict of ``expand_node_pos`` [1, M, 3], ``outcell_index`` [1, M], ``expand_node_mask``."""
    if pos.dim() != 3:
        raise ValueError("please check your pos shape: 1*N*3")
    if pos.shape[0] != 1:
        raise ValueError("sorry, we did not support pos batch size >1 in distributed version")
    p = pos[0]
    n_atoms, dev = p.shape[0], p.device
    if pbc is None:
        return {"expand_node_pos": p.unsqueeze(0),
                "outcell_index": torch.arange(n_atoms, dtype=torch.long, device=dev).unsqueeze(0),
                "expand_node_mask": torch.ones(1, n_atoms, dtype=torch.bool, device=dev)}
    periodic = [bool(v) for v in torch.as_tensor(pbc).reshape(-1)[:3]]
    steps = [range(-num_cell_perdirection, num_cell_perdirection + 1) if periodic[d] else range(0, 1)
             for d in range(3)]
    cand = torch.tensor([[i, j, k] for i in steps[0] for j in steps[1] for k in steps[2]], dtype=torch.float32,
                        device=dev)
    shift = cand @ torch.as_tensor(cell_size, dtype=torch.float32, device=dev)       # [C, 3]
    images = (p.unsqueeze(0) + shift.unsqueeze(1)).reshape(-1, 3)                   # cell-major
    lo = torch.as_tensor(cell_boundMIN, dtype=images.dtype, device=dev).reshape(1, 3)
    hi = torch.as_tensor(cell_boundMAX, dtype=images.dtype, device=dev).reshape(1, 3)
    outside = torch.clamp(torch.maximum(lo - images.detach(), images.detach() - hi), min=0.0)
    keep = torch.sqrt(torch.sum(outside ** 2, dim=-1)) < cutoff
    atom = torch.arange(n_atoms, dtype=torch.long, device=dev).repeat(cand.shape[0])
    kept = images[keep]
    return {"expand_node_pos": kept.unsqueeze(0), "outcell_index": atom[keep].unsqueeze(0),
            "expand_node_mask": torch.ones(1, kept.shape[0], dtype=torch.bool, device=dev)}


# ------------------------------------------------------------------------------------------------
# Radius graph
# ------------------------------------------------------------------------------------------------
class _DistFn(torch.autograd.Function):
    """|v| with a precomputed, bit-exact forward value and the analytic backward v/|v|."""

    @staticmethod
    def forward(ctx, vec, dist):
        ctx.save_for_backward(vec, dist)
        return dist

    @staticmethod
    def backward(ctx, g):
        vec, dist = ctx.saved_tensors
        if torch.is_grad_enabled():
            # create_graph=True: |v| formed again from v so that v/|v| is differentiable in v
            dist = torch.linalg.vector_norm(vec, dim=-1)
        safe = torch.where(dist > 0, dist, torch.ones_like(dist))
        gv = torch.where((dist > 0).unsqueeze(-1), vec * (g / safe).unsqueeze(-1), torch.zeros_like(vec))
        return gv, None


def morton_row_order(pos, cell_size):
    """Rows sorted by the Morton code of their ``cell_size`` grid cell (int32 [N])."""
    if pos.shape[0] == 0:
        return torch.zeros(0, dtype=torch.int32, device=pos.device)
    p = pos.detach().to(torch.float32)
    c = torch.floor((p - p.min(dim=0).values) / cell_size).to(torch.int64).clamp_(0, 1023)

    def spread(x):
        x = (x | (x << 16)) & 0x030000FF
        x = (x | (x << 8)) & 0x0300F00F
        x = (x | (x << 4)) & 0x030C30C3
        x = (x | (x << 2)) & 0x09249249
        return x

    code = spread(c[:, 0]) | (spread(c[:, 1]) << 1) | (spread(c[:, 2]) << 2)
    return torch.argsort(code, stable=True).to(torch.int32)


def radius_graph(pos, pts, q_ptr, p_ptr, max_dist, min_dist=-1.0, max_neighbors=None, with_key_csr=True,
                 poly_cutoff=None):
    """Flattened radius graph between queries ``pos`` [N,3] and expanded points ``pts`` [N2,3].

    ``q_ptr`` / ``p_ptr`` (int64, [B+1]) delimit the systems.  Returns a dict with the reference's
    keys (``query_idx``, ``neighbor_idx``, ``metadata``, ``f_edge_vec``, ``f_dist``, ``f_poly_dist``)
    plus ``row_order`` (spatial processing order) and ``query_sorted`` = True."""
    require_cuda(pos, pts)
    lib = _lib.load()
    dev = pos.device
    import ctypes
    p32 = pos.detach().to(torch.float32).contiguous()
    x32 = pts.detach().to(torch.float32).contiguous()
    q_ptr = torch.as_tensor(q_ptr, dtype=torch.int64).to(dev).contiguous()
    p_ptr = torch.as_tensor(p_ptr, dtype=torch.int64).to(dev).contiguous()
    NQ, P, B = p32.shape[0], x32.shape[0], q_ptr.numel() - 1
    maxnb = -1 if max_neighbors is None else int(max_neighbors)
    ws = _ws(lib.e2a_radius_graph_workspace_bytes(NQ, P, B), dev)
    E = ctypes.c_int64(0)
    C = ctypes.c_int64(0)
    st = stream_of(dev)
    check(lib.e2a_radius_graph_plan(ptr(p32), ptr(x32), ptr(q_ptr), ptr(p_ptr), NQ, P, B, float(max_dist),
                                    float(min_dist), maxnb, ctypes.byref(E), ctypes.byref(C), ptr(ws), ws.numel(),
                                    st), "e2a_radius_graph_plan")
    E, C = int(E.value), int(C.value)
    fws = _ws(lib.e2a_radius_graph_fill_workspace_bytes(C), dev)
    query_idx = torch.empty(E, dtype=torch.int64, device=dev)
    neighbor_idx = torch.empty(E, dtype=torch.int64, device=dev)
    row_ptr = torch.empty(NQ + 1, dtype=torch.int32, device=dev)
    col = torch.empty(E, dtype=torch.int32, device=dev)
    vec_k = torch.empty((E, 3), dtype=torch.float32, device=dev)
    dist_k = torch.empty(E, dtype=torch.float32, device=dev)
    poly_k = torch.empty(E, dtype=torch.float32, device=dev)
    check(lib.e2a_radius_graph_fill(ptr(p32), ptr(x32), ptr(q_ptr), ptr(p_ptr), NQ, P, B, float(max_dist),
                                    float(min_dist), maxnb, E, C, ptr(query_idx), ptr(neighbor_idx), ptr(row_ptr),
                                    ptr(col), ptr(vec_k), ptr(dist_k), ptr(poly_k), ptr(ws), ws.numel(), ptr(fws),
                                    fws.numel(), st), "e2a_radius_graph_fill")
    if with_key_csr:
        md = prepare_sparse_qk_edge_index_metadata(query_idx, neighbor_idx, NQ, P)
    else:
        md = (row_ptr, col, torch.arange(E, dtype=torch.int32, device=dev), None, None, None)
    # differentiable geometry with the kernel's bit-exact values
    vec = pos.to(torch.float32)[query_idx] - pts.to(torch.float32)[neighbor_idx]
    dist = _DistFn.apply(vec, dist_k)
    poly = polynomial(dist, float(max_dist if poly_cutoff is None else poly_cutoff))
    return {
        "query_idx": query_idx,
        "neighbor_idx": neighbor_idx,
        "metadata": md,
        "f_edge_vec": vec,
        "f_dist": dist,
        "f_poly_dist": poly,
        "row_order": morton_row_order(pos, max(float(max_dist), 1e-3)),
        "key_order": morton_row_order(pts, max(float(max_dist), 1e-3)),
        "query_sorted": True,
    }


def construct_radius_neighbor(node_pos, node_mask, expand_node_pos, expand_node_mask, max_dist,
                              include_mask=None, min_dist=-1, max_neighbors=None, error_check=False,
                              poly="poly", toy_config=None):
    """The reference's padded-batch API (module_utils.py:3119-3242): ``node_pos`` [B,L,3],
    ``node_mask`` [B,L], ``expand_node_pos`` [B,L2,3], ``expand_node_mask`` [B,L2] (valid expanded
    nodes form a prefix of each row).  ``neighbor_idx`` indexes the flattened valid expanded nodes."""
    if include_mask is not None or poly != "poly" or toy_config is not None:
        raise NotImplementedError("only the default neighbour mode (no include_mask, poly='poly') is built")
    pos = node_pos[node_mask]
    pts = expand_node_pos[expand_node_mask]
    q_ptr = torch.nn.functional.pad(node_mask.sum(-1).cumsum(0), (1, 0))
    p_ptr = torch.nn.functional.pad(expand_node_mask.sum(-1).cumsum(0), (1, 0))
    return radius_graph(pos, pts, q_ptr, p_ptr, max_dist, min_dist, max_neighbors)
