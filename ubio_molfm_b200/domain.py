"""Spatial domain decomposition of one periodic system over ranks, with a per-layer halo exchange.

Each rank owns the atoms of one slab of the cell along its first lattice vector (fractional
coordinate 0) and evaluates the energy of its own atoms.  Its graph has queries only for owned atoms;
the keys are every atom (any periodic image) within the cutoff of an owned atom: owned atoms plus
*ghosts* owned by other ranks.  Node features of the ghosts change every layer, so before every block
the ghost rows of the residual stream are refreshed from their owners (``all_to_all`` over NCCL):
the per-layer halo exchange.  The exchange is an autograd
function whose backward sends the ghosts' gradients back to their owners and adds them there, so
``E_rank.backward()`` on every rank gives exact forces on the owned atoms for the total energy
(positions go through the same exchange).  Nothing else is communicated except the final energy sum.

The result equals the single-GPU evaluation up to fp32 summation order
(``tests/test_domain.py``; the host-side logic is tested on CPU ``gloo`` ranks).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib, ops
from .graph import _DistFn, morton_row_order, pbc_image_cells, radius_graph
from .nn import polynomial


def slab_owner(pos, cell, world):
    """Owner rank of each atom: the slab of its fractional coordinate along the first lattice vector."""
    cell = torch.as_tensor(cell, dtype=torch.float64, device=pos.device)
    frac = pos.detach().to(torch.float64) @ torch.linalg.inv(cell)
    f0 = torch.remainder(frac[:, 0], 1.0)
    return torch.clamp((f0 * world).floor().to(torch.int64), 0, world - 1)


class HaloPlan:
    """Who sends which owned rows to whom.  ``local`` rows = owned atoms (ascending global id), then
    ghosts grouped by owner rank (ascending global id within an owner)."""

    def __init__(self, own_gid, ghost_gid, ghost_owner, world, rank, group=None):
        self.world, self.rank, self.group = world, rank, group
        self.n_own = own_gid.numel()
        dev = own_gid.device
        order = torch.argsort(ghost_owner * (int(ghost_gid.max()) + 1 if ghost_gid.numel() else 1) + ghost_gid)
        self.ghost_gid = ghost_gid[order]
        self.ghost_owner = ghost_owner[order]
        self.recv_counts = torch.bincount(self.ghost_owner, minlength=world).cpu()
        # requests: tell each owner how many and which of its atoms this rank needs
        cdev = dev if dist.get_backend(group) == "nccl" else torch.device("cpu")
        counts_out = torch.empty(world, dtype=torch.int64, device=cdev)
        dist.all_to_all_single(counts_out, self.recv_counts.to(cdev), group=group)
        self.send_counts = counts_out.cpu()
        req = torch.empty(int(self.send_counts.sum()), dtype=torch.int64, device=cdev)
        dist.all_to_all_single(req, self.ghost_gid.to(cdev).contiguous(), output_split_sizes=self.send_counts.tolist(),
                               input_split_sizes=self.recv_counts.tolist(), group=group)
        req = req.to(dev)
        # requested global ids -> rows of this rank's owned block
        pos_in_own = torch.searchsorted(own_gid, req)
        if req.numel() and not bool((own_gid[pos_in_own.clamp(max=max(self.n_own - 1, 0))] == req).all()):
            raise RuntimeError("halo plan: a rank requested an atom it does not own here")
        self.send_idx = pos_in_own

    def exchange(self, x_own):
        """Rows [n_own + n_ghost, ...]: owned rows, then the ghosts' current rows from their owners."""
        return _HaloFn.apply(x_own, self)


class HaloStats:
    """Opt-in timing of the halo exchanges (CUDA events around each ``all_to_all`` on the current
    stream) and of each evaluation's graph build (``"graph_build"``: the slab graph, the halo plan and
    the local neighbour dict, including the positions' exchange): ``records`` holds (what, start, end,
    bytes sent); :meth:`summary` sums them."""

    def __init__(self):
        self.enabled = False
        self.records = []

    def _start(self):
        if not self.enabled or not torch.cuda.is_available():
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def _stop(self, direction, e0, nbytes):
        if e0 is None:
            return
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record()
        self.records.append((direction, e0, e1, nbytes))

    def summary(self):
        torch.cuda.synchronize()
        out = {}
        for d, e0, e1, nb in self.records:
            o = out.setdefault(d, {"calls": 0, "ms": 0.0, "bytes": 0})
            o["calls"] += 1
            o["ms"] += e0.elapsed_time(e1)
            o["bytes"] += int(nb)
        return out


HALO_STATS = HaloStats()


class _HaloFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x_own, plan):
        send = x_own[plan.send_idx].contiguous()
        tail = tuple(x_own.shape[1:])
        recv = x_own.new_empty((int(plan.recv_counts.sum()),) + tail)
        t0 = HALO_STATS._start()
        dist.all_to_all_single(recv, send, output_split_sizes=plan.recv_counts.tolist(),
                               input_split_sizes=plan.send_counts.tolist(), group=plan.group)
        HALO_STATS._stop("forward", t0, send.numel() * send.element_size())
        ctx.plan = plan
        return torch.cat([x_own, recv], dim=0)

    @staticmethod
    def backward(ctx, g):
        plan = ctx.plan
        g = g.contiguous()
        g_own = g[:plan.n_own].clone()
        g_ghost = g[plan.n_own:].contiguous()
        back = g.new_empty((int(plan.send_counts.sum()),) + tuple(g.shape[1:]))
        t0 = HALO_STATS._start()
        dist.all_to_all_single(back, g_ghost, output_split_sizes=plan.send_counts.tolist(),
                               input_split_sizes=plan.recv_counts.tolist(), group=plan.group)
        HALO_STATS._stop("adjoint", t0, g_ghost.numel() * g_ghost.element_size())
        if back.shape[0]:
            g_own.index_add_(0, plan.send_idx, back)
        return g_own, None


def slab_keys(pos_all, own_gid, cell, pbc, cutoff):
    """Candidate keys of this rank's radius search without expanding the whole system: the periodic
    images (cell shift k, atom a) whose fractional coordinates lie inside the owned atoms' fractional
    bounding box widened by the cutoff (as a perpendicular distance per lattice direction, plus a small
    margin).  Every image within the cutoff of an owned atom is among them.

    Returns ``(index [K'] int64, cell_shift [K'] int64, atom [K'] int64, offsets [K,3] fp32)`` with
    ``index = k * N + a`` ascending: the order of :func:`~ubio_molfm_b200.graph.expand_pbc`'s images (its
    compaction keeps this order), so a search over these keys finds the same neighbours in the same
    order as one over the whole expansion."""
    dev = pos_all.device
    n = pos_all.shape[0]
    cells, offsets = pbc_image_cells(torch.as_tensor(cell, dtype=torch.float32), list(pbc), cutoff)
    cell64 = torch.as_tensor(cell, dtype=torch.float64).cpu()
    inv = torch.linalg.inv(cell64)
    delta = (float(cutoff) * torch.linalg.norm(inv, dim=0) + 1e-6).to(dev)          # per lattice direction
    frac = pos_all.detach().to(torch.float64) @ inv.to(dev)                             # [N, 3]
    own = frac[own_gid]
    lo, hi = own.min(dim=0).values - delta, own.max(dim=0).values + delta
    f_img = frac.unsqueeze(0) + cells.to(dev, torch.float64).unsqueeze(1)              # [K, N, 3]
    inside = ((f_img >= lo) & (f_img <= hi)).all(dim=-1)
    index = torch.nonzero(inside.reshape(-1)).flatten()
    return index, index // n, index % n, offsets.to(dev)


def domain_graph(pos_all, cell, pbc, cutoff, max_neighbors, world, rank, group=None):
    """Graph of this rank's owned atoms over the owned + ghost atoms, and the halo plan.

    Returns ``(plan, own_gid, local_gid, geometry)``; ``geometry`` holds the local expanded nodes
    (``outcell`` into local rows, image ``offsets``), the edge list (queries = owned local rows,
    neighbours = local expanded nodes) and the kernel's bit-exact distances."""
    dev = pos_all.device
    owner = slab_owner(pos_all, cell, world)
    own_gid = torch.nonzero(owner == rank).flatten()
    n_own = own_gid.numel()
    p = pos_all.detach().to(torch.float32)
    # keys: the images near the owned atoms only (the same neighbours, in the same order, as a search
    # over the whole system's expansion)
    _, image_g, outcell_g, offsets = slab_keys(p, own_gid, cell, pbc, cutoff)
    keys = p[outcell_g] + offsets[image_g]
    g = radius_graph(p[own_gid], keys, torch.tensor([0, n_own]), torch.tensor([0, keys.shape[0]]), cutoff,
                     1e-4, max_neighbors, with_key_csr=False)
    used = torch.unique(g["neighbor_idx"])                                   # candidate keys used (sorted)
    atoms_needed = torch.unique(outcell_g[used])
    is_own = torch.zeros(pos_all.shape[0], dtype=torch.bool, device=dev)
    is_own[own_gid] = True
    ghost_gid = atoms_needed[~is_own[atoms_needed]]
    plan = HaloPlan(own_gid, ghost_gid, owner[ghost_gid], world, rank, group)
    local_gid = torch.cat([own_gid, plan.ghost_gid])
    g2l = torch.full((pos_all.shape[0],), -1, dtype=torch.int64, device=dev)
    g2l[local_gid] = torch.arange(local_gid.numel(), device=dev)
    e2l = torch.full((keys.shape[0],), -1, dtype=torch.int64, device=dev)
    e2l[used] = torch.arange(used.numel(), device=dev)
    geometry = {
        "outcell": g2l[outcell_g[used]],
        "offsets": offsets[image_g[used]],
        "query_idx": g["query_idx"],
        "neighbor_idx": e2l[g["neighbor_idx"]],
        "dist": g["f_dist"].detach(),
    }
    return plan, own_gid, local_gid, geometry


def local_graph(pos_local, geometry, n_local, cutoff, n_query=None):
    """The decoder's neighbour dict on the local rows, differentiable in ``pos_local``.  With ``n_query``
    (the owned atoms, the leading rows) only those rows are queries: the ghosts that follow them serve
    as keys and values only, and the decoder computes nothing else for them."""
    nq = n_local if n_query is None else int(n_query)
    outcell, qi, ni = geometry["outcell"], geometry["query_idx"], geometry["neighbor_idx"]
    exp_pos = pos_local[outcell] + geometry["offsets"]
    vec = pos_local[qi] - exp_pos[ni]
    dist_ = _DistFn.apply(vec, geometry["dist"])
    md = ops.prepare_sparse_qk_edge_index_metadata(qi, ni, nq, exp_pos.shape[0])
    g = {
        "query_idx": qi, "neighbor_idx": ni, "metadata": md, "f_edge_vec": vec, "f_dist": dist_,
        "f_poly_dist": polynomial(dist_, float(cutoff)), "f_outcell_index": outcell, "f_exp_node_pos": exp_pos,
        "row_order": morton_row_order(pos_local[:nq], max(float(cutoff), 1e-3)),
        "key_order": morton_row_order(exp_pos, max(float(cutoff), 1e-3)), "query_sorted": True,
    }
    if nq != n_local:
        g["n_query"] = nq
    return g


def domain_energy_forces(model, pos_all, Z_all, cell, pbc=(True, True, True), group=None, charge=None,
                         multiplicity=None):
    """Energy of the whole system and forces on this rank's owned atoms under slab decomposition.

    ``pos_all`` / ``Z_all``: every atom's position and type (replicated on every rank).  ``charge`` /
    ``multiplicity``: the system's (one value each, or None), whose embedding every row takes, ghosts
    included.  Returns ``(energy_total [1], own_gid, forces_own [n_own, 3])``; every rank must call it
    (collectives)."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    dec = model.decoder
    t0 = HALO_STATS._start()
    plan, own_gid, local_gid, geom = domain_graph(pos_all, cell, pbc, dec.max_radius, dec.max_neighbors, world,
                                                  rank, group)
    with torch.enable_grad():
        pos_own = pos_all.detach()[own_gid].to(torch.float32).requires_grad_(True)
        pos_local = plan.exchange(pos_own)
        graph = local_graph(pos_local, geom, local_gid.numel(), dec.max_radius, n_query=plan.n_own)
        HALO_STATS._stop("graph_build", t0, 0)
        sys_emb = None
        if charge is not None:
            mult = torch.ones(1, dtype=torch.long) if multiplicity is None else multiplicity
            sys_emb = model.backbone.system_embedding(charge, mult)[:1]
        # the ghosts' key / value projections come from their owners (no norm or projection work here
        # for atoms owned elsewhere)
        x = dec(pos_local, Z_all[local_gid], graph, True, kv_halo=lambda t, which: plan.exchange(t),
                sys_embedding=sys_emb)
        e_own = model.energy_head(x[:plan.n_own, 0]).squeeze(-1).sum()
        (grad,) = torch.autograd.grad(e_own, pos_own)
    if pos_own.is_cuda and model.check_device_status:
        _lib.raise_on_device_status(pos_own.device)
    energy = e_own.detach().reshape(1).clone()
    dist.all_reduce(energy, group=group)
    return energy, own_gid, -grad


# ------------------------------------------------------------------------------------------------
# Config 4: independent molecules, data parallel
# ------------------------------------------------------------------------------------------------
def shard_molecules(sizes, world):
    """Balanced assignment of molecules to ranks: largest first, each to the rank with the fewest atoms
    so far (ties to the lower rank).  Returns one sorted index list per rank."""
    order = sorted(range(len(sizes)), key=lambda i: (-int(sizes[i]), i))
    load = [0] * world
    out = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += int(sizes[i])
    return [sorted(v) for v in out]


def molecules_energy_forces(model, mols, device, max_atoms_per_call=60000):
    """Energies [M] and forces (list of [n_i, 3]) of non-periodic molecules ``mols`` = [(pos, Z) or
    (pos, Z, charge, multiplicity), ...], evaluated in batches of at most ``max_atoms_per_call`` atoms
    (systems never see each other).  With charges given, each molecule's charge / multiplicity system
    embedding enters its evaluation (e2former_wrapper.py:249-259)."""
    energies, forces = [], []
    with_charge = len(mols) > 0 and len(mols[0]) >= 4
    i = 0
    while i < len(mols):
        j, n = i, 0
        while j < len(mols) and (j == i or n + len(mols[j][1]) <= max_atoms_per_call):
            n += len(mols[j][1])
            j += 1
        part = mols[i:j]
        pos = torch.cat([torch.as_tensor(m[0], dtype=torch.float32) for m in part]).to(device)
        Z = torch.cat([torch.as_tensor(m[1], dtype=torch.int64) for m in part]).to(device)
        batch = torch.cat([torch.full((len(m[1]),), k, dtype=torch.int64) for k, m in enumerate(part)]).to(device)
        kw = {}
        if with_charge:
            kw = {"charge": torch.tensor([int(m[2]) for m in part]), "multiplicity": torch.tensor([int(m[3]) for m in part])}
        e, f = model(pos, Z, None, (False, False, False), batch, **kw)
        energies.append(e)
        forces.extend(torch.split(f, [len(m[1]) for m in part]))
        i = j
    return torch.cat(energies), forces


def gather_molecule_results(energies, forces, idx, n_total, group=None, dst=0):
    """Every rank's molecule energies and forces on rank ``dst``, ordered by molecule index.

    ``energies`` [m_r], ``forces`` a list of [n_i, 3] in the order of ``idx`` (this rank's molecule
    indices).  One size exchange, then one gather of a padded buffer per rank holding, per molecule,
    its index, atom count and energy, followed by all its forces.  Returns ``(energies [n_total],
    [forces of molecule 0, 1, ...])`` on ``dst`` and ``(None, None)`` elsewhere."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    dev = energies.device
    m = len(idx)
    sizes = [int(f.shape[0]) for f in forces]
    n_words = 3 * m + 3 * sum(sizes)
    cnt = torch.tensor([n_words, m], device=dev, dtype=torch.int64)
    all_cnt = [torch.zeros_like(cnt) for _ in range(world)]
    dist.all_gather(all_cnt, cnt, group=group)
    all_cnt = [c.tolist() for c in all_cnt]
    width = max(c[0] for c in all_cnt)
    buf = torch.zeros(max(width, 1), device=dev, dtype=torch.float64)
    if m:
        head = torch.stack([torch.as_tensor(idx, dtype=torch.float64, device=dev),
                            torch.tensor(sizes, dtype=torch.float64, device=dev), energies.to(torch.float64)], 1)
        buf[:3 * m] = head.reshape(-1)
        if sum(sizes):
            buf[3 * m:n_words] = torch.cat([f.reshape(-1) for f in forces]).to(torch.float64)
    bufs = [torch.zeros_like(buf) for _ in range(world)] if rank == dst else None
    dist.gather(buf, bufs, dst=dst, group=group)
    if rank != dst:
        return None, None
    out_e = torch.zeros(n_total, device=dev, dtype=energies.dtype)
    out_f = [None] * n_total
    for b, (words, k) in zip(bufs, all_cnt):
        if k == 0:
            continue
        hd = b[:3 * k].reshape(k, 3)
        mol = hd[:, 0].long()
        nat = hd[:, 1].long().tolist()
        out_e[mol] = hd[:, 2].to(energies.dtype)
        fl = b[3 * k:words].reshape(-1, 3).to(energies.dtype)
        for j, part in zip(mol.tolist(), torch.split(fl, nat)):
            out_f[j] = part
    return out_e, out_f
