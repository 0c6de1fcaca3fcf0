"""GPU-resident molecular dynamics around ``E2FormerPotential``.

Mirrors the reference's torch-native MD stack (interface/ase/torch_ext/), without ASE:

* :class:`TorchAtoms` -- the tensor-backed atoms object of torch_atoms.py:15-140: positions, momenta,
  masses, cell and pbc live on the device in ``dtype`` (float64 by default, torch_atoms.py:34), with
  the same getters / setters (``get_positions``, ``set_positions``, ``get_velocities``,
  ``get_momenta``, ``set_momenta``, ``get_forces(md=True, copy=False)``, ``get_potential_energy``)
  and an attached calculator.
* :class:`E2FormerCalculator` -- the TorchAtoms fast path of the reference calculator
  (ase/calculator/e2former_calculator.py:143-197): the model is evaluated in float32 on the current
  positions with the system's charge and multiplicity, results are cached until the positions change
  and returned in the atoms' dtype (``add_ref_energy`` adds per-element reference energies).
* :class:`TorchLangevin` -- torch_langevin.py:96-281: the Vanden-Eijnden--Ciccotti Langevin scheme
  (c1 = dt/2 - dt^2 fr/8, c2 = dt fr/2 - dt^2 fr^2/8, noise terms c3..c5); with ``friction=0`` it is
  exactly velocity Verlet (NVE), and the noise draw is skipped.  ``fixcm`` re-centres the momenta
  after each step with ``TorchFixCom`` (torch_constraints.py:70-76); a ``"FixCom"`` constraint on the
  atoms also re-centres positions and projects the noise.
* :class:`VelocityVerlet` -- a convenience NVE driver on the same classes.

ASE units throughout: positions in Angstrom, energies in eV, masses in amu, time in
Angstrom sqrt(amu / eV) (``FS`` of them per femtosecond, from the CODATA 2014 constants ASE uses).
Every tensor stays on the GPU; the only host work per step is the graph build's size query.
"""
from __future__ import annotations

import math

import torch

_E_CHARGE = 1.6021766208e-19      # C   (CODATA 2014)
_AMU = 1.660539040e-27            # kg  (CODATA 2014)
FS = 1e-15 * 1e10 * math.sqrt(_E_CHARGE / _AMU)   # ASE time units per femtosecond
KB_EV = 8.6173303e-5              # eV / K (CODATA 2014)


class TorchAtoms:
    """Atoms whose state is device tensors (torch_atoms.py:15-140).  ``numbers`` [N] ints, ``positions``
    [N,3], ``masses`` [N] (amu; required: the element table of ASE is not restated here), ``cell`` [3,3]
    or None, ``pbc`` 3 bools, ``momenta`` [N,3] or None.  ``constraints``: a list that may hold
    ``"FixCom"`` (ASE's FixCom constraint, torch_constraints.py:55-95), applied by ``set_positions`` /
    ``set_momenta`` before the new values are stored (torch_atoms.py:431-470)."""

    def __init__(self, numbers, positions, masses, cell=None, pbc=(False, False, False), momenta=None,
                 device="cuda", dtype=torch.float64, charge=0, multiplicity=1):
        self._device, self._dtype = torch.device(device), dtype
        self._torch_numbers = torch.as_tensor(numbers).to(self._device, torch.long)
        self._torch_positions = torch.as_tensor(positions).to(self._device, dtype).clone()
        self._torch_masses = torch.as_tensor(masses).to(self._device, dtype)
        self._torch_momenta = (torch.zeros_like(self._torch_positions) if momenta is None
                               else torch.as_tensor(momenta).to(self._device, dtype).clone())
        self._torch_cell = None if cell is None else torch.as_tensor(cell).to(self._device, dtype)
        # the model's graph build takes the cell on the host: kept there too (no device read per step)
        self._cell_host = None if cell is None else torch.as_tensor(cell).detach().to("cpu", torch.float32)
        self.pbc = tuple(bool(p) for p in pbc)
        self.charge, self.multiplicity = int(charge), int(multiplicity)
        self._torch_forces = None
        self.calc = None
        self.constraints = []

    def __len__(self):
        return self._torch_positions.shape[0]

    def get_positions(self):
        return self._torch_positions

    def set_positions(self, positions, apply_constraint=True):
        positions = positions.to(self._device, self._dtype)
        if apply_constraint and "FixCom" in self.constraints:
            positions = _fixcom_positions(self, positions)
        self._torch_positions = positions

    def get_momenta(self):
        return self._torch_momenta

    def set_momenta(self, momenta, apply_constraint=True):
        momenta = momenta.to(self._device, self._dtype)
        if apply_constraint and "FixCom" in self.constraints:
            momenta = _fixcom_momenta(self, momenta)
        self._torch_momenta = momenta

    def get_velocities(self):
        return self._torch_momenta / self._torch_masses.unsqueeze(-1)

    def set_velocities(self, velocities):
        self.set_momenta(velocities.to(self._device, self._dtype) * self._torch_masses.unsqueeze(-1))

    def get_masses(self):
        return self._torch_masses

    def get_cell(self):
        return self._torch_cell

    def get_forces(self, md=False, copy=True):
        if self.calc is None:
            raise RuntimeError("TorchAtoms has no calculator attached")
        f = self.calc.get_forces(self)
        return f.clone() if copy else f

    def get_potential_energy(self):
        if self.calc is None:
            raise RuntimeError("TorchAtoms has no calculator attached")
        return self.calc.get_potential_energy(self)

    def get_kinetic_energy(self):
        return 0.5 * (self._torch_momenta * self._torch_momenta / self._torch_masses.unsqueeze(-1)).sum()

    def get_temperature(self, fixed_com=True):
        """Instantaneous temperature (K) with 3N - 3 degrees of freedom when the COM is fixed."""
        dof = 3 * len(self) - (3 if fixed_com else 0)
        return 2.0 * self.get_kinetic_energy() / (dof * KB_EV)


class E2FormerCalculator:
    """Energy / forces of a :class:`TorchAtoms` from a potential ``(pos fp32, Z, cell, pbc, batch,
    charge=, multiplicity=) -> (energy [1], forces [N,3])`` (e2former_calculator.py:143-197, the
    TorchAtoms backend).  Cached until the positions tensor is replaced or modified in place (its
    identity and version counter: no device sync); outputs in the atoms' dtype."""

    def __init__(self, potential, ref_energy=None, add_ref_energy=True, use_charge=True):
        self.potential = potential
        self.ref_energy = ref_energy
        self.add_ref_energy = add_ref_energy
        self.use_charge = use_charge
        self._key = None
        self.results = {}

    def _evaluate(self, atoms):
        x = atoms.get_positions()
        if self._key is not None and self._key[0] is x and self._key[1] == x._version:
            return
        kw = {}
        if self.use_charge:
            kw = {"charge": torch.tensor([atoms.charge]), "multiplicity": torch.tensor([atoms.multiplicity])}
        energy, forces = self.potential(x.to(torch.float32), atoms._torch_numbers, atoms._cell_host, atoms.pbc, **kw)
        energy = energy.reshape(-1)[0].to(atoms._dtype)
        if self.add_ref_energy and self.ref_energy is not None:
            energy = energy + torch.as_tensor(self.ref_energy, device=x.device,
                                              dtype=atoms._dtype)[atoms._torch_numbers].sum()
        self.results = {"energy": energy, "forces": forces.to(atoms._dtype)}
        self._key = (x, x._version)

    def get_forces(self, atoms):
        self._evaluate(atoms)
        return self.results["forces"]

    def get_potential_energy(self, atoms):
        self._evaluate(atoms)
        return self.results["energy"]


def _fixcom_positions(atoms, new_x):
    """TorchFixCom.adjust_positions (torch_constraints.py:58-68)."""
    m = atoms.get_masses()
    ms = m.sum()
    old_cm = (m.unsqueeze(-1) * atoms.get_positions()).sum(0) / ms
    new_cm = (m.unsqueeze(-1) * new_x).sum(0) / ms
    return new_x + (old_cm - new_cm)


def _fixcom_momenta(atoms, p):
    """TorchFixCom.adjust_momenta (torch_constraints.py:70-76)."""
    m = atoms.get_masses()
    return p - m.unsqueeze(-1) * (p.sum(0) / m.sum())


def _fixcom_noise(atoms, f):
    """TorchFixCom.adjust_forces (torch_constraints.py:78-95): removes the mass-weighted mean."""
    m = atoms.get_masses()
    lmd = (m.unsqueeze(-1) * f).sum(0) / m.square().sum()
    return f - m.unsqueeze(-1) * lmd


class TorchLangevin:
    """torch_langevin.py:96-281.  ``timestep`` in ASE time units, ``temperature_K`` the bath
    temperature, ``friction`` in inverse ASE time units (0 = NVE velocity Verlet)."""

    def __init__(self, atoms, timestep, temperature_K=0.0, friction=None, fixcm=True, rng=None):
        if friction is None:
            raise TypeError("Missing required 'friction' argument.")
        self.atoms, self.dt, self.fr = atoms, float(timestep), float(friction)
        self.temp = KB_EV * float(temperature_K)
        self.fix_com = fixcm
        self._rng = rng
        self.nsteps = 0
        self.updatevars()

    def updatevars(self):
        a, dt, T, fr = self.atoms, self.dt, self.temp, self.fr
        m = a.get_masses()
        self._inv_m = (1.0 / m).unsqueeze(-1)
        sigma = torch.sqrt((2.0 * T * fr) / m)
        self._deterministic = fr == 0.0
        self.c1 = dt / 2.0 - dt * dt * fr / 8.0
        self.c2 = dt * fr / 2.0 - dt * dt * fr * fr / 8.0
        self._c3 = math.sqrt(dt) * sigma / 2.0 - dt ** 1.5 * fr * sigma / 8.0
        self._c5 = dt ** 1.5 * sigma / (2.0 * math.sqrt(3.0))
        self._c4 = fr / 2.0 * self._c5

    def set_temperature(self, temperature_K):
        self.temp = KB_EV * float(temperature_K)
        self.updatevars()

    def step(self, forces=None):
        a = self.atoms
        f = a.get_forces(md=True, copy=False) if forces is None else forces.to(a._device, a._dtype)
        v = a.get_velocities()
        x = a.get_positions()
        if self._deterministic:
            rnd_pos = rnd_vel = None
        else:
            xi = torch.randn(x.shape, generator=self._rng, device=x.device, dtype=x.dtype)
            eta = torch.randn(x.shape, generator=self._rng, device=x.device, dtype=x.dtype)
            if "FixCom" in a.constraints:
                xi, eta = _fixcom_noise(a, xi), _fixcom_noise(a, eta)
            rnd_pos = eta * self._c5.unsqueeze(-1)
            rnd_vel = xi * self._c3.unsqueeze(-1) - eta * self._c4.unsqueeze(-1)
        v_half = v + (self.c1 * f * self._inv_m - self.c2 * v)
        if rnd_vel is not None:
            v_half = v_half + rnd_vel
        x_new = x + self.dt * v_half
        if rnd_pos is not None:
            x_new = x_new + rnd_pos
        a.set_positions(x_new, apply_constraint=True)
        # with ``fixcm`` (and no FixCom constraint) the reference re-centres the positions after storing
        # them, against the stored ones (torch_langevin.py:229-235 with torch_constraints.py:58-68): the
        # shift is zero, so the positions are left as they are here; only the momenta are re-centred
        x_new = a.get_positions()
        f_new = a.get_forces(md=True, copy=False)
        disp = x_new - x if rnd_pos is None else x_new - x - rnd_pos
        v = disp / self.dt
        v = v + (self.c1 * f_new * self._inv_m - self.c2 * v)
        if rnd_vel is not None:
            v = v + rnd_vel
        p = v * a.get_masses().unsqueeze(-1)
        a.set_momenta(p, apply_constraint=True)
        if self.fix_com and "FixCom" not in a.constraints:
            a.set_momenta(_fixcom_momenta(a, a.get_momenta()), apply_constraint=False)
        self.nsteps += 1
        return f_new

    def run(self, steps):
        for _ in range(steps):
            self.step()


class VelocityVerlet:
    """NVE driver: ``potential(pos, Z, cell, pbc, ...) -> (energy [1], forces [N,3])`` on
    :class:`TorchAtoms` / :class:`E2FormerCalculator` / :class:`TorchLangevin` (friction 0), with the
    state (``x``, ``v``, ``f``, ``energy``) in ``dtype`` (float64 by default, as the reference keeps
    it); the potential sees float32 positions."""

    def __init__(self, potential, pos, atomic_numbers, masses, cell, pbc, dt_fs=0.5, velocities=None, fix_com=True,
                 dtype=torch.float64, charge=None, multiplicity=None):
        dev = pos.device
        self.atoms = TorchAtoms(atomic_numbers, pos, masses, cell, pbc, device=dev, dtype=dtype,
                                charge=0 if charge is None else charge,
                                multiplicity=1 if multiplicity is None else multiplicity)
        self.atoms.calc = E2FormerCalculator(potential, use_charge=charge is not None)
        if velocities is not None:
            self.atoms.set_velocities(torch.as_tensor(velocities))
        if fix_com:
            self.atoms.set_momenta(_fixcom_momenta(self.atoms, self.atoms.get_momenta()))
        self.integrator = TorchLangevin(self.atoms, float(dt_fs) * FS, friction=0.0, fixcm=fix_com)
        self.dt = self.integrator.dt
        self.fix_com = fix_com
        self.m = self.atoms.get_masses()

    @property
    def x(self):
        return self.atoms.get_positions()

    @property
    def v(self):
        return self.atoms.get_velocities()

    @property
    def f(self):
        return self.atoms.get_forces(md=True, copy=False)

    @property
    def energy(self):
        return self.atoms.get_potential_energy().reshape(1)

    @property
    def nsteps(self):
        return self.integrator.nsteps

    def _com(self, x):
        return (self.m.unsqueeze(-1) * x).sum(0) / self.m.sum()

    def step(self):
        self.integrator.step()
        return self.energy

    def run(self, steps):
        for _ in range(steps):
            self.step()
        return self.energy

    def kinetic_energy(self):
        return self.atoms.get_kinetic_energy()

    def temperature(self):
        return self.atoms.get_temperature(self.fix_com)


def maxwell_boltzmann(masses, temperature_K, generator=None, device="cpu", dtype=torch.float64):
    """Velocities (ASE units) drawn from the Maxwell-Boltzmann distribution at ``temperature_K``."""
    m = torch.as_tensor(masses, dtype=torch.float64)
    sigma = torch.sqrt(KB_EV * float(temperature_K) / m).unsqueeze(-1)
    v = torch.randn((m.shape[0], 3), generator=generator, dtype=torch.float64) * sigma
    return v.to(dtype).to(device)
