"""Seeded synthetic systems and seeded parameters for benchmarks and parity tests.

The reference benchmarks on public datasets that are not available here; these generators build
seeded stand-ins with the shapes, sizes and value distributions of the named workloads:

* :func:`water_box` -- rigid H2O on a cubic lattice with jitter and random orientations
  (216 molecules / 18.64 A box for the 648-atom water workload).
* :func:`uniform_box` -- positions uniform in a periodic cube sized for an average of ``k``
  neighbours within ``cutoff`` (the attention-layer microbenchmark graphs).
* :func:`bio_box` -- H/C/N/O/S mixture at a target mass density with a minimum interatomic
  distance (rejection sampling on a cell grid).
* :func:`molecule_batch` -- non-periodic random-tree conformers for batched inference.

:func:`seeded_params_` overwrites every trainable floating-point parameter of a module with values
drawn from a generator seeded by ``(seed, parameter name)``.  Because the draw depends only on the
name and shape, two modules with the reference's ``state_dict`` layout receive identical weights.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np
import torch

MASS = {1: 1.008, 6: 12.011, 7: 14.007, 8: 15.999, 9: 18.998, 16: 32.06, 17: 35.45}
AVOGADRO = 6.02214076e23


def _rng(seed):
    return np.random.default_rng(seed)


def random_rotations(rng, n):
    """Uniform random rotation matrices (via normalised quaternions)."""
    q = rng.normal(size=(n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q.T
    return np.stack([
        np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)], -1),
        np.stack([2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)], -1),
        np.stack([2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)], -1),
    ], 1)


def water_box(n_side=6, box=18.64, jitter=0.3, seed=0):
    """Rigid water (O-H 0.9572 A, H-O-H 104.52 deg) on an ``n_side``^3 lattice in a cubic PBC box.

    Returns ``(pos [N,3] float64, Z [N] int64, cell [3,3] float64)`` with atoms ordered O,H,H per
    molecule.
    """
    rng = _rng(seed)
    spacing = box / n_side
    g = (np.arange(n_side) + 0.5) * spacing
    centres = np.stack(np.meshgrid(g, g, g, indexing="ij"), -1).reshape(-1, 3)
    centres = centres + rng.uniform(-jitter, jitter, size=centres.shape)
    th = math.radians(104.52) / 2
    r = 0.9572
    local = np.array([[0.0, 0.0, 0.0], [r * math.sin(th), r * math.cos(th), 0.0],
                      [-r * math.sin(th), r * math.cos(th), 0.0]])
    rot = random_rotations(rng, len(centres))
    pos = centres[:, None, :] + np.einsum("nij,aj->nai", rot, local)
    pos = np.mod(pos.reshape(-1, 3), box)
    Z = np.tile(np.array([8, 1, 1]), len(centres))
    return pos, Z, np.eye(3) * box


def uniform_box_side(n_atoms, k_avg, cutoff=6.0):
    """Cube side giving an average of ``k_avg`` neighbours within ``cutoff`` at uniform density."""
    return (n_atoms * (4.0 / 3.0) * math.pi * cutoff ** 3 / k_avg) ** (1.0 / 3.0)


def uniform_box(n_atoms, k_avg, cutoff=6.0, seed=0, elements=(1, 6, 7, 8)):
    """Positions uniform in a periodic cube with ~``k_avg`` neighbours within ``cutoff``."""
    rng = _rng(seed)
    side = uniform_box_side(n_atoms, k_avg, cutoff)
    pos = rng.uniform(0.0, side, size=(n_atoms, 3))
    Z = rng.choice(np.array(elements), size=n_atoms)
    return pos, Z, np.eye(3) * side


def _poisson_fill(rng, n_atoms, side, dmin, inside=None, max_tries=200):
    """Rejection sampling on a hash grid: ``n_atoms`` points in [0,side)^3, min distance ``dmin``."""
    ncell = max(1, int(side // dmin))
    h = side / ncell
    grid = {}
    pts = []
    tries = 0
    while len(pts) < n_atoms:
        tries += 1
        if tries > max_tries * n_atoms:
            raise RuntimeError("rejection sampling did not converge; lower density or dmin")
        p = rng.uniform(0.0, side, size=3)
        if inside is not None and not inside(p):
            continue
        c = tuple((p // h).astype(int) % ncell)
        ok = True
        for dx in (-1, 0, 1):
            for dy in (-1, 0, 1):
                for dz in (-1, 0, 1):
                    cc = ((c[0] + dx) % ncell, (c[1] + dy) % ncell, (c[2] + dz) % ncell)
                    for q in grid.get(cc, ()):
                        d = p - q
                        d -= side * np.round(d / side)
                        if d @ d < dmin * dmin:
                            ok = False
                            break
                    if not ok:
                        break
                if not ok:
                    break
            if not ok:
                break
        if ok:
            grid.setdefault(c, []).append(p)
            pts.append(p)
    return np.array(pts)


def bio_box(n_atoms=1500, density=1.0, dmin=0.9, seed=0,
            fractions=((1, 0.50), (6, 0.30), (7, 0.08), (8, 0.11), (16, 0.01))):
    """H/C/N/O/S mixture at ``density`` g/cm^3 in a periodic cube, min distance ``dmin``."""
    rng = _rng(seed)
    els = np.array([e for e, _ in fractions])
    fr = np.array([f for _, f in fractions])
    counts = np.floor(fr / fr.sum() * n_atoms).astype(int)
    counts[0] += n_atoms - counts.sum()
    Z = np.repeat(els, counts)
    rng.shuffle(Z)
    mass_g = sum(MASS[int(z)] for z in Z) / AVOGADRO
    side = (mass_g / density * 1e24) ** (1.0 / 3.0)
    pos = _poisson_fill(rng, n_atoms, side, dmin)
    return pos, Z, np.eye(3) * side


def blob_in_water(box=100.0, n_blob=8000, blob_density=1.35, water_density=1.0, dmin=0.9, jitter=0.3, seed=0,
                  fractions=((1, 0.50), (6, 0.30), (7, 0.08), (16, 0.01), (8, 0.11))):
    """Large periodic system: a spherical H/C/N/O/S blob of ``n_blob`` atoms at ``blob_density``
    (g/cm^3, min distance ``dmin``) in the centre of a cubic box of rigid water at ``water_density``
    (molecules on a jittered lattice with random orientations; molecules whose oxygen lies within the
    blob radius + 1.5 A are left out).  About 1e5 atoms at the defaults."""
    rng = _rng(seed)
    els = np.array([e for e, _ in fractions])
    fr = np.array([f for _, f in fractions])
    counts = np.floor(fr / fr.sum() * n_blob).astype(int)
    counts[0] += n_blob - counts.sum()
    Zb = np.repeat(els, counts)
    rng.shuffle(Zb)
    mass_g = sum(MASS[int(z)] for z in Zb) / AVOGADRO
    radius = (3.0 * mass_g / blob_density * 1e24 / (4.0 * math.pi)) ** (1.0 / 3.0)
    side = 2.0 * radius
    centre = np.full(3, side / 2.0)
    pb = _poisson_fill(rng, n_blob, side, dmin, inside=lambda p: np.linalg.norm(p - centre) <= radius)
    pb = pb - centre + box / 2.0
    # water lattice at the requested density
    mol_mass_g = (MASS[8] + 2 * MASS[1]) / AVOGADRO
    spacing = (mol_mass_g / water_density * 1e24) ** (1.0 / 3.0)
    n_side = max(1, int(round(box / spacing)))
    g = (np.arange(n_side) + 0.5) * (box / n_side)
    centres = np.stack(np.meshgrid(g, g, g, indexing="ij"), -1).reshape(-1, 3)
    centres = centres + rng.uniform(-jitter, jitter, size=centres.shape)
    keep = np.linalg.norm(centres - box / 2.0, axis=1) > radius + 1.5
    centres = centres[keep]
    th = math.radians(104.52) / 2
    r = 0.9572
    local = np.array([[0.0, 0.0, 0.0], [r * math.sin(th), r * math.cos(th), 0.0],
                      [-r * math.sin(th), r * math.cos(th), 0.0]])
    rot = random_rotations(rng, len(centres))
    pw = (centres[:, None, :] + np.einsum("nij,aj->nai", rot, local)).reshape(-1, 3)
    Zw = np.tile(np.array([8, 1, 1]), len(centres))
    pos = np.mod(np.concatenate([pb, pw], axis=0), box)
    Z = np.concatenate([Zb, Zw])
    return pos, Z, np.eye(3) * box


def molecule_batch(n_mol, min_atoms=10, max_atoms=60, seed=0,
                   elements=(1, 6, 7, 8, 9, 16, 17)):
    """Non-periodic random-tree conformers: bonds 1.0-1.6 A with +-0.05 A noise, seeded.

    Returns a list of ``(pos [n,3], Z [n], charge, multiplicity)``.
    """
    rng = _rng(seed)
    out = []
    for _ in range(n_mol):
        n = int(rng.integers(min_atoms, max_atoms + 1))
        pos = np.zeros((n, 3))
        for i in range(1, n):
            for _try in range(100):
                parent = int(rng.integers(0, i))
                d = rng.normal(size=3)
                d /= np.linalg.norm(d)
                bond = rng.uniform(1.0, 1.6) + rng.uniform(-0.05, 0.05)
                p = pos[parent] + bond * d
                if i == 1 or np.min(np.linalg.norm(pos[:i] - p, axis=1)) > 0.95:
                    break
            pos[i] = p
        Z = rng.choice(np.array(elements), size=n)
        out.append((pos, Z, int(rng.integers(-1, 2)), 1))
    return out


# ------------------------------------------------------------------------------------------------
# Seeded parameters
# ------------------------------------------------------------------------------------------------
_FROZEN_SUFFIXES = ("selected_idx", "CG_weight", "path_norm", "expand_index", "sum_vec", "offset")


def _name_seed(seed, name):
    h = hashlib.sha256(f"{seed}:{name}".encode()).digest()
    return int.from_bytes(h[:8], "little") & ((1 << 63) - 1)


def seeded_tensor(seed, name, shape, kind="weight"):
    """Deterministic CPU float32 tensor for parameter ``name`` (independent of module layout)."""
    g = torch.Generator().manual_seed(_name_seed(seed, name))
    u = torch.rand(shape, generator=g, dtype=torch.float64) * 2.0 - 1.0
    if kind == "norm":
        return (1.0 + 0.1 * u).float()
    if kind == "bias":
        return (0.1 * u).float()
    fan_in = shape[-1] if len(shape) >= 2 else max(1, shape[0])
    return (u / math.sqrt(fan_in)).float()


# fixtures with a charge / multiplicity: the system embedding tables drawn 300x larger and its linear 3x, so that the
# embedding moves energies and forces well beyond the parity tolerances
SYSTEM_EMBED_GAINS = {"embedding_charge.": 300.0, "embedding_multiplicity.": 300.0, "mix_cm.": 3.0}


def seeded_params_(module: torch.nn.Module, seed: int = 0, gains=None):
    """Overwrite trainable float parameters of ``module`` in place (frozen tables are kept).
    ``gains``: {parameter-name prefix: factor} applied after the draw (e.g. to make a small term of
    the model large enough for a test to see)."""
    with torch.no_grad():
        for name, p in module.named_parameters():
            if not p.is_floating_point() or name.endswith(_FROZEN_SUFFIXES) or not p.requires_grad:
                continue
            if ".Jd_list." in name or name.startswith("Jd_list"):
                continue
            leaf = name.rsplit(".", 1)[-1]
            if p.dim() == 1 and leaf == "weight":
                kind = "norm"
            elif leaf.startswith("bias") or (p.dim() == 1):
                kind = "bias"
            elif "embedding" in name:
                kind = "bias"
            else:
                kind = "weight"
            t = seeded_tensor(seed, name, tuple(p.shape), kind)
            for pre, f in (gains or {}).items():
                if name.startswith(pre):
                    t = t * f
            p.copy_(t.to(p.device))
    return module
