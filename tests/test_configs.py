"""The reference's CPU-runnable configurations as parity cases on the GPU: the CUDA model against the
CPU oracle (``oracle/model_ref.py`` on graphs from the C graph oracle), same seeded weights by
parameter name.

* config 1: 216 rigid waters (648 atoms) in an 18.64 A periodic box, small model (32 channels per
  degree, 8 heads, 32 basis functions, 4 layers, cutoff 5 A, no neighbour cap): energy and forces,
  then 10 NVE velocity-Verlet steps at 0.5 fs from seeded Maxwell-Boltzmann velocities at 300 K, the
  CUDA trajectory against the same integrator driven by the oracle's forces;
* config 3: a 1,500-atom H/C/N/O/S box at 1.0 g/cm^3, full-size model (256 channels per degree, 128
  heads, 256 basis functions, 4 layers, cutoff 4.5 A, <= 32 neighbours): energy and forces.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"

SMALL = dict(irreps_node_embedding="32x0e+32x1e+32x2e", num_layers=4, max_neighbors=None, max_radius=5.0,
             number_of_basis=32, num_attn_heads=8, attn_scalar_head=8, irreps_head="4x0e+4x1e+4x2e",
             norm_layer="rms_norm_sh", alpha_drop=0.0, tp_type="QK_alpha", attn_type="so2-first-order",
             atom_type_cnt=256, avg_degree=23.0)
FULL = dict(SMALL, irreps_node_embedding="256x0e+256x1e+256x2e", max_neighbors=32, max_radius=4.5,
            number_of_basis=256, num_attn_heads=128, irreps_head="2x0e+2x1e+2x2e")


def _models(cfg, seed):
    from ubio_molfm_b200.model import E2FormerPotential
    from ubio_molfm_b200.synthetic import seeded_params_

    m = E2FormerPotential(**cfg)
    seeded_params_(m.decoder, seed)
    seeded_params_(m.energy_head, seed + 1)
    p = {k: v.detach().clone() for k, v in m.decoder.state_dict().items()}
    ph = {k: v.detach().clone() for k, v in m.energy_head.state_dict().items()}
    return m.to(DEV).eval(), p, ph


def _oracle_potential(p, ph, cfg, cell):
    """CPU potential (pos, Z, cell, pbc) -> (energy [1], forces) from the oracles."""
    from oracle import graph_ref
    from oracle import model_ref as M
    from ubio_molfm_b200.graph import pbc_image_offsets

    off = pbc_image_offsets(np.asarray(cell), [True, True, True], cfg["max_radius"]).numpy()

    def pot(pos, Z, _cell=None, _pbc=None):
        x = pos.detach().cpu().float()
        pn = x.numpy()
        n = len(pn)
        ia = graph_ref.pbc_expand(pn, off, cfg["max_radius"])
        outcell, offsets = ia % n, off[ia // n]
        exp = (pn[outcell] + offsets).astype(np.float32)
        qi, ni, _ = graph_ref.radius_graph(pn, exp, [0, n], [0, len(exp)], cfg["max_radius"], 1e-4,
                                           cfg["max_neighbors"])
        graph = (torch.tensor(qi), torch.tensor(ni), torch.tensor(outcell), torch.tensor(offsets), True)
        e, f, _ = M.energy_forces(p, ph, cfg, x, Z.detach().cpu(), graph)
        return e, f

    return pot


def _check_energy_forces(energy, forces, e_ref, f_ref, n_atoms):
    de = abs(float(energy.sum()) - float(e_ref.sum())) / n_atoms
    assert de <= 1e-6 * abs(float(e_ref.sum())) / n_atoms + 1e-7, (float(energy.sum()), float(e_ref.sum()))
    assert (forces.detach().cpu().double() - f_ref.double()).abs().max().item() <= 1e-4


def test_config1_water648_energy_forces_and_nve():
    from ubio_molfm_b200.md import VelocityVerlet, maxwell_boltzmann
    from ubio_molfm_b200.synthetic import MASS, water_box

    model, p, ph = _models(SMALL, 11)
    pos, Z, cell = water_box(n_side=6, box=18.64, jitter=0.3, seed=1)
    pos_t, Z_t = torch.tensor(pos, dtype=torch.float32), torch.tensor(Z)
    cell_t = torch.tensor(cell, dtype=torch.float32)
    pbc = (True, True, True)
    oracle = _oracle_potential(p, ph, SMALL, cell)
    energy, forces = model(pos_t.to(DEV), Z_t.to(DEV), cell_t, pbc)
    e_ref, f_ref = oracle(pos_t, Z_t)
    _check_energy_forces(energy, forces, e_ref, f_ref, len(Z))

    masses = [MASS[int(z)] for z in Z]
    v0 = maxwell_boltzmann(masses, 300.0, torch.Generator().manual_seed(3))
    md_gpu = VelocityVerlet(model, pos_t.to(DEV), Z_t.to(DEV), masses, cell_t, pbc, dt_fs=0.5, velocities=v0.to(DEV))
    md_cpu = VelocityVerlet(oracle, pos_t.clone(), Z_t, masses, cell_t, pbc, dt_fs=0.5, velocities=v0.clone())
    for _ in range(10):
        md_gpu.step()
        md_cpu.step()
    assert md_gpu.nsteps == md_cpu.nsteps == 10
    _check_energy_forces(md_gpu.energy, md_gpu.f, md_cpu.energy, md_cpu.f, len(Z))
    # both integrators keep float64 state (as the reference's TorchAtoms does); they differ only by the
    # forces, which agree to the fp32 force tolerance (1e-4 eV/A) at each step
    assert md_gpu.x.dtype == md_cpu.x.dtype == torch.float64
    assert (md_gpu.x.cpu() - md_cpu.x).abs().max().item() <= 1e-6
    assert (md_gpu.v.cpu() - md_cpu.v).abs().max().item() <= 1e-4


def test_config3_bio1500_full_model_energy_forces():
    from ubio_molfm_b200.synthetic import bio_box

    model, p, ph = _models(FULL, 13)
    pos, Z, cell = bio_box(n_atoms=1500, density=1.0, dmin=0.9, seed=4)
    pos_t, Z_t = torch.tensor(pos, dtype=torch.float32), torch.tensor(Z)
    cell_t = torch.tensor(cell, dtype=torch.float32)
    energy, forces = model(pos_t.to(DEV), Z_t.to(DEV), cell_t, (True, True, True))
    e_ref, f_ref = _oracle_potential(p, ph, FULL, cell)(pos_t, Z_t)
    _check_energy_forces(energy, forces, e_ref, f_ref, len(Z))


def test_use_faiss_order_equals_default():
    """``use_faiss=True`` (the expanded-node order of the reference's FAISS path) changes only the index
    space of the expanded nodes: energy and forces equal the default expansion's on the config-1 box."""
    from ubio_molfm_b200.model import E2FormerPotential
    from ubio_molfm_b200.synthetic import seeded_params_, water_box

    pos, Z, cell = water_box(n_side=6, box=18.64, jitter=0.3, seed=1)
    pos_t, Z_t = torch.tensor(pos, dtype=torch.float32, device=DEV), torch.tensor(Z, device=DEV)
    cell_t = torch.tensor(cell, dtype=torch.float32)
    out = []
    for faiss_order in (False, True):
        m = E2FormerPotential(use_faiss=faiss_order, **SMALL)
        seeded_params_(m.decoder, 11)
        seeded_params_(m.energy_head, 12)
        m = m.to(DEV).eval()
        out.append(m(pos_t, Z_t, cell_t, (True, True, True)))
        g, _ = m.build_graph(pos_t, cell_t, (True, True, True), None)
        out[-1] = out[-1] + (g["query_idx"].numel(),)
    (e0, f0, n0), (e1, f1, n1) = out
    assert n0 == n1
    _check_energy_forces(e1, f1, e0.detach().cpu(), f0.detach().cpu(), len(Z))


def test_config5_like_blob_in_water_full_model_cutoff6():
    """Config 5's composition and cutoff at a size the CPU oracle finishes: a seeded 1,000-atom
    H/C/N/O/S blob at 1.35 g/cm^3 in rigid water at 1.0 g/cm^3 (40 A periodic cube, ~6k atoms), the
    full-size model at cutoff 6 A with <= 32 neighbours: energy and forces against the oracle."""
    from ubio_molfm_b200.synthetic import blob_in_water

    cfg = dict(FULL, max_radius=6.0)
    model, p, ph = _models(cfg, 17)
    pos, Z, cell = blob_in_water(box=40.0, n_blob=1000, seed=5)
    assert 5000 <= len(Z) <= 10000
    pos_t, Z_t = torch.tensor(pos, dtype=torch.float32), torch.tensor(Z)
    cell_t = torch.tensor(cell, dtype=torch.float32)
    energy, forces = model(pos_t.to(DEV), Z_t.to(DEV), cell_t, (True, True, True))
    e_ref, f_ref = _oracle_potential(p, ph, cfg, cell)(pos_t, Z_t)
    _check_energy_forces(energy, forces, e_ref, f_ref, len(Z))
