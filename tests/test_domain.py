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
    allE = gather_molecule_results(energies, mine, len(sizes))
    out[rank] = allE.tolist() == [float(10 * i + 1) for i in range(len(sizes))]
    dist.destroy_process_group()


def test_gather_molecule_results_gloo():
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_gather_worker, args=(3, _free_port(), out), nprocs=3, join=True)
    assert all(out[r] for r in range(3)), dict(out)
