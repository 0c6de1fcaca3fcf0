"""GPU-resident NVE molecular dynamics around ``E2FormerPotential`` (velocity Verlet).

The deterministic path of the reference's ``TorchLangevin`` (interface/ase/torch_ext/torch_langevin.py:
185-281 with friction 0: c1 = dt/2, c2 = 0, no noise), with ``TorchFixCom``
(torch_constraints.py:55-76) keeping the centre of mass fixed:

    v_half = v + (dt/2) F / m
    x'     = x + dt v_half               (+ the centre-of-mass shift back to its old place)
    F'     = F(x')
    v'     = (x' - x) / dt + (dt/2) F' / m   (- the centre-of-mass velocity)

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


class VelocityVerlet:
    """NVE integrator.  ``potential(pos, Z, cell, pbc) -> (energy [1], forces [N,3])``."""

    def __init__(self, potential, pos, atomic_numbers, masses, cell, pbc, dt_fs=0.5, velocities=None, fix_com=True):
        dev = pos.device
        self.potential, self.Z, self.cell, self.pbc = potential, atomic_numbers, cell, pbc
        self.x = pos.detach().to(torch.float32).clone()
        self.m = torch.as_tensor(masses, dtype=torch.float32, device=dev)
        self.inv_m = (1.0 / self.m).unsqueeze(-1)
        self.dt = float(dt_fs) * FS
        self.v = (torch.zeros_like(self.x) if velocities is None
                  else torch.as_tensor(velocities, dtype=torch.float32, device=dev).clone())
        self.fix_com = fix_com
        if fix_com:
            self.v = self._remove_com_velocity(self.v)
        self.energy, self.f = self.potential(self.x, self.Z, self.cell, self.pbc)
        self.nsteps = 0

    def _com(self, x):
        return (self.m.unsqueeze(-1) * x).sum(0) / self.m.sum()

    def _remove_com_velocity(self, v):
        p = self.m.unsqueeze(-1) * v
        return v - p.sum(0) / self.m.sum()

    def step(self):
        x_old = self.x
        v_half = self.v + (0.5 * self.dt) * self.f * self.inv_m
        x_new = x_old + self.dt * v_half
        if self.fix_com:
            x_new = x_new + (self._com(x_old) - self._com(x_new))
        self.energy, self.f = self.potential(x_new, self.Z, self.cell, self.pbc)
        v = (x_new - x_old) / self.dt + (0.5 * self.dt) * self.f * self.inv_m
        self.v = self._remove_com_velocity(v) if self.fix_com else v
        self.x = x_new
        self.nsteps += 1
        return self.energy

    def run(self, steps):
        for _ in range(steps):
            self.step()
        return self.energy

    def kinetic_energy(self):
        return 0.5 * (self.m.unsqueeze(-1) * self.v * self.v).sum()

    def temperature(self):
        """Instantaneous temperature (K) with 3N - 3 degrees of freedom when the COM is fixed."""
        dof = 3 * self.x.shape[0] - (3 if self.fix_com else 0)
        return 2.0 * self.kinetic_energy() / (dof * KB_EV)


def maxwell_boltzmann(masses, temperature_K, generator=None, device="cpu"):
    """Velocities (ASE units) drawn from the Maxwell-Boltzmann distribution at ``temperature_K``."""
    m = torch.as_tensor(masses, dtype=torch.float64)
    sigma = torch.sqrt(KB_EV * float(temperature_K) / m).unsqueeze(-1)
    v = torch.randn((m.shape[0], 3), generator=generator, dtype=torch.float64) * sigma
    return v.to(torch.float32).to(device)
