"""The MD stack's host logic (TorchAtoms / calculator / TorchLangevin) on CPU with an analytic
potential: float64 state, the velocity-Verlet update of the reference's zero-friction Langevin
scheme (interface/ase/torch_ext/torch_langevin.py:20-62, 192-281), FixCom, and the Langevin noise path."""
import torch

from ubio_molfm_b200.md import FS, E2FormerCalculator, TorchAtoms, TorchLangevin, VelocityVerlet


def _harmonic(k=2.0):
    def pot(pos, Z, cell=None, pbc=None, **kw):
        x = pos.double()
        e = 0.5 * k * (x * x).sum()
        return e.reshape(1).float(), (-k * x).float()
    return pot


def test_velocity_verlet_float64_state_matches_hand_rolled_update():
    g = torch.Generator().manual_seed(0)
    n = 12
    x0 = torch.randn(n, 3, generator=g, dtype=torch.float64) * 3 + 50.0
    v0 = torch.randn(n, 3, generator=g, dtype=torch.float64) * 0.01
    m = torch.rand(n, generator=g, dtype=torch.float64) * 10 + 1
    pot = _harmonic()
    md = VelocityVerlet(pot, x0.clone(), torch.ones(n, dtype=torch.long), m, None, (False,) * 3, dt_fs=0.5,
                        velocities=v0.clone(), fix_com=False)
    assert md.x.dtype == torch.float64 and md.v.dtype == torch.float64
    x, v, dt = x0.clone(), v0.clone(), 0.5 * FS
    f = pot(x.float(), None)[1].double()
    for _ in range(5):
        md.step()
        xn = x + dt * (v + 0.5 * dt * f / m[:, None])
        fn = pot(xn.float(), None)[1].double()
        v = (xn - x) / dt + 0.5 * dt * fn / m[:, None]
        x, f = xn, fn
    assert torch.allclose(md.x, x, rtol=0, atol=1e-12)
    assert torch.allclose(md.v, v, rtol=0, atol=1e-10)


def test_nve_energy_conservation_and_fixcom():
    g = torch.Generator().manual_seed(1)
    n = 30
    x0 = torch.randn(n, 3, generator=g, dtype=torch.float64)
    x0 = x0 - x0.mean(0)                      # equal masses, centre at the well's minimum: the total force
    v0 = torch.randn(n, 3, generator=g, dtype=torch.float64) * 0.05
    v0 = v0 - v0.mean(0)                      # stays zero, so re-centring the momenta takes no energy
    m = torch.full((n,), 4.0, dtype=torch.float64)
    atoms = TorchAtoms(torch.ones(n), x0, m, device="cpu")
    atoms.set_velocities(v0)
    atoms.calc = E2FormerCalculator(_harmonic(0.5), use_charge=False)
    dyn = TorchLangevin(atoms, 0.5 * FS, friction=0.0, fixcm=True)
    e0 = float(atoms.get_potential_energy() + atoms.get_kinetic_energy())
    for _ in range(200):
        dyn.step()
    e1 = float(atoms.get_potential_energy() + atoms.get_kinetic_energy())
    assert abs(e1 - e0) < 1e-4 * abs(e0)
    assert atoms.get_momenta().sum(0).abs().max().item() < 1e-12       # momenta re-centred every step
    assert dyn.nsteps == 200


def test_fixcom_constraint_and_langevin_noise_path():
    g = torch.Generator().manual_seed(2)
    n = 16
    m = torch.rand(n, generator=g, dtype=torch.float64) + 1
    atoms = TorchAtoms(torch.ones(n), torch.randn(n, 3, generator=g, dtype=torch.float64), m, device="cpu")
    atoms.constraints = ["FixCom"]
    atoms.calc = E2FormerCalculator(_harmonic(1.0), use_charge=False)
    com0 = (m[:, None] * atoms.get_positions()).sum(0) / m.sum()
    dyn = TorchLangevin(atoms, 0.5 * FS, temperature_K=300.0, friction=0.01, fixcm=False,
                        rng=torch.Generator().manual_seed(3))
    for _ in range(50):
        dyn.step()
    com1 = (m[:, None] * atoms.get_positions()).sum(0) / m.sum()
    assert (com1 - com0).abs().max().item() < 1e-12
    assert atoms.get_momenta().sum(0).abs().max().item() < 1e-12
    assert float(atoms.get_kinetic_energy()) > 0.0


def test_calculator_caches_until_positions_change():
    calls = []

    def pot(pos, Z, cell=None, pbc=None, **kw):
        calls.append(kw)
        return torch.zeros(1), torch.zeros_like(pos)

    atoms = TorchAtoms([1, 8], torch.zeros(2, 3), [1.0, 16.0], device="cpu", charge=-1, multiplicity=2)
    atoms.calc = E2FormerCalculator(pot)
    atoms.get_forces()
    atoms.get_potential_energy()
    assert len(calls) == 1 and int(calls[0]["charge"]) == -1 and int(calls[0]["multiplicity"]) == 2
    atoms.get_positions().add_(0.1)        # in-place change
    atoms.get_forces()
    atoms.set_positions(atoms.get_positions() + 0.1)
    atoms.get_forces()
    assert len(calls) == 3
