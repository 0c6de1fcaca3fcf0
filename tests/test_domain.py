"""Domain decomposition: the halo exchange on CPU gloo ranks; the full model on 2 GPUs."""
import os
import socket
import subprocess
import sys

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _halo_worker(rank, world, port, out):
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from ubio_molfm_b200.domain import HaloPlan

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n = 23
    owner = torch.arange(n) % world
    g = torch.Generator().manual_seed(0)
    need = torch.rand(world, n, generator=g) < 0.5          # rank r needs atom a as a ghost
    own = torch.nonzero(owner == rank).flatten()
    ghost = torch.nonzero(need[rank] & (owner != rank)).flatten()
    plan = HaloPlan(own, ghost, owner[ghost], world, rank)
    feat = torch.arange(n, dtype=torch.float64).unsqueeze(1) * torch.tensor([[1.0, -2.0]], dtype=torch.float64)
    x_own = feat[own].clone().requires_grad_(True)
    y = plan.exchange(x_own)
    local = torch.cat([own, plan.ghost_gid])
    ok_fwd = torch.equal(y.detach(), feat[local])
    w = torch.rand(world, n, 2, generator=torch.Generator().manual_seed(1), dtype=torch.float64)
    (y * w[rank][local]).sum().backward()
    # d/dx_a of sum_r sum_{local rows of r} w[r, a] y = w[owner, a] + sum_{r needs a} w[r, a]
    expect = w[rank][own].clone()
    for r in range(world):
        if r != rank:
            m = need[r][own]
            expect[m] += w[r][own][m]
    out[rank] = (ok_fwd, torch.allclose(x_own.grad, expect))
    dist.destroy_process_group()


def _halo_fault_worker(rank, world, port, out):
    """Rank ``world - 1`` leaves after the plan is built (a rank that died between steps); the others
    must get an error from their next exchange within the process group's timeout instead of waiting."""
    import datetime
    import time

    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from ubio_molfm_b200.domain import HaloPlan

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    n = 12
    owner = torch.arange(n) % world
    own = torch.nonzero(owner == rank).flatten()
    ghost = torch.nonzero(owner != rank).flatten()        # every other atom is a ghost
    plan = HaloPlan(own, ghost, owner[ghost], world, rank)
    if rank == world - 1:
        out[rank] = "left"
        return                                            # leaves without exchanging (no teardown)
    t0 = time.monotonic()
    try:
        plan.exchange(torch.ones(own.numel(), 2))
        out[rank] = "no error"
    except RuntimeError:
        out[rank] = "error after %.1f s" % (time.monotonic() - t0)


def test_halo_exchange_reports_a_missing_rank_gloo():
    mgr = mp.Manager()
    out = mgr.dict()
    world = 3
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_halo_fault_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert out.get(world - 1) == "left", dict(out)
    for r in range(world - 1):
        assert str(out.get(r, "")).startswith("error after"), dict(out)
        assert float(str(out[r]).split()[2]) < 30.0, dict(out)


@pytest.mark.parametrize("world", [2, 3])
def test_halo_exchange_forward_and_adjoint_gloo(world):
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_halo_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    assert all(out[r] == (True, True) for r in range(world)), dict(out)


def test_slab_owner_partitions_periodic_cell():
    from ubio_molfm_b200.domain import slab_owner

    cell = torch.tensor([[10.0, 0, 0], [1.0, 8.0, 0], [0.5, 0.5, 9.0]])
    frac = torch.rand(500, 3, generator=torch.Generator().manual_seed(3)) * 3 - 1   # outside [0,1) too
    pos = frac @ cell
    own = slab_owner(pos, cell, 4)
    expect = (torch.remainder(frac[:, 0].double(), 1.0) * 4).floor().long()
    assert torch.equal(own, expect.clamp(0, 3))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_slab_keys_cover_every_neighbour(world):
    """The keys a rank's radius search sees (slab_keys) include every periodic image within the cutoff
    of any atom it owns, in a triclinic cell with stored positions outside the home cell, in the
    expansion's (cell shift, atom) order."""
    from ubio_molfm_b200.domain import slab_keys, slab_owner
    from ubio_molfm_b200.graph import pbc_image_cells

    g = torch.Generator().manual_seed(7)
    cell = torch.tensor([[30.0, 0, 0], [4.0, 25.0, 0], [2.0, 3.0, 28.0]])
    pos = (torch.rand(400, 3, generator=g) * 1.4 - 0.2) @ cell
    cutoff = 5.0
    cells, offsets = pbc_image_cells(cell, [True] * 3, cutoff)
    exp_pos = (pos.unsqueeze(0) + offsets.unsqueeze(1)).reshape(-1, 3)   # every candidate image, k * N + a
    owner = slab_owner(pos, cell, world)
    for rank in range(world):
        own_gid = torch.nonzero(owner == rank).flatten()
        index, image, atom, off = slab_keys(pos, own_gid, cell, [True] * 3, cutoff)
        assert torch.equal(index, image * pos.shape[0] + atom) and bool(torch.all(index[1:] > index[:-1]))
        assert torch.equal(off, offsets)
        near = (torch.cdist(pos[own_gid].double(), exp_pos.double()) <= cutoff).any(0)
        need = torch.nonzero(near).flatten()
        assert bool(torch.isin(need, index).all())
        assert index.numel() < exp_pos.shape[0]


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 8])
def test_domain_graph_edges_equal_whole_system_search(world, monkeypatch):
    """A rank's edges from the slab keys equal, edge for edge and in order (query, neighbour position,
    distance bit for bit), those of a radius search of its owned atoms over the whole system's PBC
    expansion."""
    from ubio_molfm_b200 import domain
    from ubio_molfm_b200.graph import expand_pbc, radius_graph
    from ubio_molfm_b200.synthetic import blob_in_water

    pos_np, _, cell = blob_in_water(box=40.0, n_blob=1000, seed=5)
    pos = torch.tensor(pos_np, dtype=torch.float32, device="cuda")
    monkeypatch.setattr(domain, "HaloPlan", _LocalPlan)
    for rank in (0, world - 1):
        plan, own_gid, local_gid, geom = domain.domain_graph(pos, cell, (True,) * 3, 6.0, 32, world, rank)
        pos_local = pos[local_gid]
        key_pos = pos_local[geom["outcell"]] + geom["offsets"]
        exp_pos, _, _ = expand_pbc(pos, torch.tensor(cell, dtype=torch.float32), [True] * 3, 6.0)
        ref = radius_graph(pos[own_gid], exp_pos, torch.tensor([0, own_gid.numel()]),
                           torch.tensor([0, exp_pos.shape[0]]), 6.0, 1e-4, 32, with_key_csr=False)
        assert torch.equal(geom["query_idx"], ref["query_idx"])
        assert torch.equal(key_pos[geom["neighbor_idx"]], exp_pos[ref["neighbor_idx"]])
        assert torch.equal(geom["dist"], ref["f_dist"].detach())


@pytest.mark.gpu
def test_domain_decomposition_equals_single_gpu():
    """2 ranks over NCCL (when the box has 2 GPUs): energy and forces of the slab-decomposed model
    equal the single-GPU evaluation (fp32 summation order only)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "domain_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT,
                         env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "DOMAIN_OK" in res.stdout, res.stdout[-3000:]


class _LocalPlan:
    """HaloPlan stand-in without collectives: the same ordering of the ghost rows."""

    def __init__(self, own_gid, ghost_gid, ghost_owner, world, rank, group=None):
        self.n_own = own_gid.numel()
        order = torch.argsort(ghost_owner * (int(ghost_gid.max()) + 1 if ghost_gid.numel() else 1) + ghost_gid)
        self.ghost_gid = ghost_gid[order]


@pytest.mark.gpu
@pytest.mark.parametrize("restrict", [True, False, "kv"])
def test_domain_slab_on_one_gpu_matches_full_system(restrict, monkeypatch):
    """One rank's slab of a 2-rank decomposition, on one GPU, with the halo exchange replaced by the
    full system's own tensors for the ghost rows: the owned atoms' per-atom energies equal the
    full-system ones, with the ghosts as keys only (``n_query`` = owned rows: no query-side, output or
    FFN work on them), with every row computed, and ("kv", what ``domain_energy_forces`` runs) with the
    ghosts' key / value projections exchanged instead of their block inputs."""
    from ubio_molfm_b200 import domain
    from ubio_molfm_b200.model import E2FormerPotential
    from ubio_molfm_b200.synthetic import bio_box, seeded_params_

    cfg = dict(irreps_node_embedding="128x0e+128x1e+128x2e", num_layers=2, max_neighbors=32, max_radius=4.5,
               number_of_basis=32, num_attn_heads=64, attn_scalar_head=8, irreps_head="2x0e+2x1e+2x2e",
               norm_layer="rms_norm_sh", alpha_drop=0.0, atom_type_cnt=256, avg_degree=23.0)
    model = E2FormerPotential(**cfg)
    seeded_params_(model.decoder, 21)
    seeded_params_(model.energy_head, 22)
    model = model.cuda().eval()
    dec = model.decoder
    pos, Z, cell = bio_box(n_atoms=900, seed=5)
    pos = torch.tensor(pos, dtype=torch.float32, device="cuda")
    Z = torch.tensor(Z, device="cuda")
    pbc = (True, True, True)

    inputs, kv = [], {"key": [], "value": []}
    hooks = [b.register_forward_pre_hook(lambda m, a, kw: inputs.append(kw["node_irreps"].detach()),
                                         with_kwargs=True) for b in dec.blocks]
    for b in dec.blocks:
        hooks.append(b.ga.key_linear.register_forward_hook(lambda m, a, o: kv["key"].append(o.detach())))
        hooks.append(b.ga.proj_value.register_forward_hook(lambda m, a, o: kv["value"].append(o.detach())))
    with torch.no_grad():
        g, pbc_any = model.build_graph(pos, torch.tensor(cell, dtype=torch.float32), pbc, None)
        x_full = dec(pos, Z, g, pbc_any)
        e_full = model.energy_head(x_full[:, 0]).squeeze(-1)
    for h in hooks:
        h.remove()
    assert len(inputs) == cfg["num_layers"]

    monkeypatch.setattr(domain, "HaloPlan", _LocalPlan)
    plan, own_gid, local_gid, geom = domain.domain_graph(pos, cell, pbc, dec.max_radius, dec.max_neighbors, 2, 0)
    assert 0 < plan.n_own < pos.shape[0] and plan.ghost_gid.numel() > 0
    step = iter(range(cfg["num_layers"]))

    def halo(t):
        return torch.cat([t[:plan.n_own], inputs[next(step)][plan.ghost_gid]], dim=0)

    calls = {"key": 0, "value": 0}

    def kv_halo(t, which):
        layer = calls[which]
        calls[which] += 1
        assert t.shape[0] == plan.n_own
        return torch.cat([t, kv[which][layer][plan.ghost_gid]], dim=0)

    with torch.no_grad():
        pos_local = pos[local_gid]
        graph = domain.local_graph(pos_local, geom, local_gid.numel(), dec.max_radius,
                                   n_query=plan.n_own if restrict else None)
        if restrict == "kv":
            x = dec(pos_local, Z[local_gid], graph, True, kv_halo=kv_halo)
            assert calls == {"key": cfg["num_layers"], "value": cfg["num_layers"]}
        else:
            x = dec(pos_local, Z[local_gid], graph, True, halo=halo)
        e_own = model.energy_head(x[:plan.n_own, 0]).squeeze(-1)
    if restrict:
        assert x.shape[0] == plan.n_own   # the blocks returned the query rows only
    ref = e_full[own_gid]
    assert (e_own - ref).abs().max().item() <= 1e-5 * ref.abs().max().item() + 1e-6


def test_shard_molecules_balances_and_partitions():
    from ubio_molfm_b200.domain import shard_molecules

    g = torch.Generator().manual_seed(9)
    sizes = torch.randint(10, 61, (4096,), generator=g).tolist()
    for world in (1, 2, 4, 8):
        parts = shard_molecules(sizes, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(sizes)))
        loads = [sum(sizes[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= 60


def _gather_worker(rank, world, port, out):
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from ubio_molfm_b200.domain import gather_molecule_results, shard_molecules

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sizes = [5, 9, 2, 7, 7, 3, 11]
    parts = shard_molecules(sizes, world)
    mine = parts[rank]
    energies = torch.tensor([float(10 * i + 1) for i in mine])
    forces = [torch.arange(3 * sizes[i], dtype=torch.float32).reshape(-1, 3) + 100 * i for i in mine]
    allE, allF = gather_molecule_results(energies, forces, mine, len(sizes))
    if rank == 0:
        ok = allE.tolist() == [float(10 * i + 1) for i in range(len(sizes))]
        ok &= all(torch.equal(allF[i], torch.arange(3 * sizes[i], dtype=torch.float32).reshape(-1, 3) + 100 * i)
                  for i in range(len(sizes)))
    else:
        ok = allE is None and allF is None
    out[rank] = ok
    dist.destroy_process_group()


def test_gather_molecule_results_gloo():
    """Energies and forces of every rank's molecules end up on rank 0 in molecule order (3 ranks; one
    rank holds fewer molecules, so the padded buffers differ in fill)."""
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_gather_worker, args=(3, _free_port(), out), nprocs=3, join=True)
    assert all(out[r] for r in range(3)), dict(out)
