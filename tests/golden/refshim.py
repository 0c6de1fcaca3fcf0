"""Test-only import shim that lets the reference E2Former-V2 sources run on CPU in this container.

TEST INFRASTRUCTURE ONLY. Nothing under ``ubio_molfm_b200/`` imports this module; it exists so
that ``make_golden.py`` can execute the reference's own pure-PyTorch attention path
(``tp_type="QK_alpha"``, no Triton) and record golden input/output vectors.

The reference imports third-party packages that are not installed here (e3nn, torch_geometric,
torch_cluster, opt_einsum_fx, faiss).  This shim registers minimal stand-ins in ``sys.modules``:

* ``e3nn.o3.Irreps`` -- parse / index / ``*`` (list repetition) / ``sort`` / ``simplify`` / ``dim``,
  restating e3nn's published semantics.
* ``e3nn.o3._wigner._su2_clebsch_gordan`` -- standard Condon-Shortley SU(2) Clebsch-Gordan
  coefficients (Racah formula, via ``sympy.physics.wigner.clebsch_gordan``), laid out
  ``[2j1+1, 2j2+1, 2j3+1]`` indexed by ``j+m`` as e3nn does.
* ``e3nn.o3._wigner.change_basis_real_to_complex`` -- e3nn's real<->complex harmonic basis change,
  including its ``(-1j)**l`` phase that makes the real CG coefficients real.
* ``e3nn.o3._spherical_harmonics._spherical_harmonics`` -- component-normalised real spherical
  harmonics for l<=2 (same polynomials as the reference's own ``sph_fromxyz``,
  ``module_utils.py:136-179``).
* ``e3nn.math.normalize2mom`` -- second-moment normaliser of an activation (constant found by
  Gauss-Hermite quadrature of E[f(z)^2], z~N(0,1)).
* no-op ``compile_mode`` and dummy classes for import-time-only symbols.

The reference package ``molfm.models.e2former`` is mounted as a bare package (its ``__init__`` is
not executed) and the off-path modules ``maceblocks``, ``wigner6j.tensor_product`` and
``wigner6j.base_tensor_product`` are replaced by stubs, so that ``e2former.py``,
``wigner6j/so2_tensor_product.py`` and ``module_utils.py`` load unmodified.
"""
from __future__ import annotations

import math
import os
import sys
import types
from collections import namedtuple

import numpy as np
import torch

# the reference: set E2A_REFERENCE_ROOT to a checkout (the directory holding ``src/molfm``) or to an
# installed copy (the directory holding ``molfm``)
REF_ROOT = os.environ.get("E2A_REFERENCE_ROOT", "")
# a checkout holds the package under src/; an installed copy (pip --target) holds it at the top
REF_SRC = (os.path.join(REF_ROOT, "src") if os.path.isdir(os.path.join(REF_ROOT, "src", "molfm"))
           else REF_ROOT)
E2F_DIR = os.path.join(REF_SRC, "molfm", "models", "e2former")


# --------------------------------------------------------------------------------------------
# e3nn.o3.Irreps
# --------------------------------------------------------------------------------------------
class Irrep(tuple):
    def __new__(cls, l, p=1):
        if isinstance(l, Irrep):
            return l
        if isinstance(l, str):
            s = l.strip()
            p = {"e": 1, "o": -1, "y": (-1) ** int(s[:-1])}[s[-1]]
            l = int(s[:-1])
        return super().__new__(cls, (int(l), int(p)))

    @property
    def l(self):
        return self[0]

    @property
    def p(self):
        return self[1]

    @property
    def dim(self):
        return 2 * self.l + 1

    def __repr__(self):
        return f"{self.l}{'e' if self.p == 1 else 'o'}"


class _MulIr(tuple):
    def __new__(cls, mul, ir):
        return super().__new__(cls, (int(mul), Irrep(ir)))

    @property
    def mul(self):
        return self[0]

    @property
    def ir(self):
        return self[1]

    @property
    def dim(self):
        return self.mul * self.ir.dim

    def __repr__(self):
        return f"{self.mul}x{self.ir}"


_SortResult = namedtuple("_SortResult", ["irreps", "p", "inv"])


class Irreps(tuple):
    def __new__(cls, irreps=None):
        if irreps is None:
            return super().__new__(cls, ())
        if isinstance(irreps, Irreps):
            return super().__new__(cls, tuple(irreps))
        out = []
        if isinstance(irreps, str):
            for part in irreps.split("+"):
                part = part.strip()
                if not part:
                    continue
                if "x" in part:
                    mul, ir = part.split("x")
                    out.append(_MulIr(int(mul), Irrep(ir)))
                else:
                    out.append(_MulIr(1, Irrep(part)))
        else:
            for item in irreps:
                if isinstance(item, _MulIr):
                    out.append(item)
                elif isinstance(item, (tuple, list)) and len(item) == 2 and not isinstance(item, Irrep):
                    out.append(_MulIr(item[0], Irrep(item[1]) if not isinstance(item[1], Irrep) else item[1]))
                else:
                    out.append(_MulIr(1, Irrep(item)))
        return super().__new__(cls, tuple(out))

    @property
    def dim(self):
        return sum(m.dim for m in self)

    @property
    def num_irreps(self):
        return sum(m.mul for m in self)

    @property
    def lmax(self):
        return max(m.ir.l for m in self)

    def __mul__(self, other):
        return Irreps(tuple(self) * int(other))

    __rmul__ = __mul__

    def __add__(self, other):
        return Irreps(tuple(self) + tuple(Irreps(other)))

    def __getitem__(self, i):
        r = tuple.__getitem__(self, i)
        return Irreps(r) if isinstance(i, slice) else r

    def sort(self):
        order = sorted(range(len(self)), key=lambda i: (self[i].ir.l, -self[i].ir.p * (-1) ** self[i].ir.l, i))
        irreps = Irreps([self[i] for i in order])
        inv = [0] * len(order)
        for new, old in enumerate(order):
            inv[old] = new
        return _SortResult(irreps, tuple(inv), tuple(order))

    def simplify(self):
        out = []
        for mul, ir in self:
            if out and out[-1][1] == ir:
                out[-1] = (out[-1][0] + mul, ir)
            elif mul > 0:
                out.append((mul, ir))
        return Irreps(out)

    def __contains__(self, ir):
        """``Irrep in Irreps`` (e3nn semantics: some block carries that irrep)."""
        try:
            ir = Irrep(ir)
        except (ValueError, KeyError, TypeError):
            return tuple.__contains__(self, ir)
        return any(m.ir == ir for m in self)

    def __repr__(self):
        return "+".join(repr(m) for m in self)


# --------------------------------------------------------------------------------------------
# Clebsch-Gordan and basis change (e3nn.o3._wigner)
# --------------------------------------------------------------------------------------------
def _su2_clebsch_gordan(j1, j2, j3):
    from sympy import Rational
    from sympy.physics.wigner import clebsch_gordan

    mat = torch.zeros((2 * j1 + 1, 2 * j2 + 1, 2 * j3 + 1), dtype=torch.float64)
    if abs(j1 - j2) <= j3 <= j1 + j2:
        for m1 in range(-j1, j1 + 1):
            for m2 in range(-j2, j2 + 1):
                m3 = m1 + m2
                if abs(m3) <= j3:
                    v = clebsch_gordan(Rational(j1), Rational(j2), Rational(j3),
                                       Rational(m1), Rational(m2), Rational(m3))
                    mat[j1 + m1, j2 + m2, j3 + m3] = float(v)
    return mat


def change_basis_real_to_complex(l, dtype=None, device=None):
    q = torch.zeros((2 * l + 1, 2 * l + 1), dtype=torch.complex128)
    s2 = 1.0 / math.sqrt(2.0)
    for m in range(-l, 0):
        q[l + m, l + abs(m)] = s2
        q[l + m, l - abs(m)] = -1j * s2
    q[l, l] = 1.0
    for m in range(1, l + 1):
        q[l + m, l + abs(m)] = (-1) ** m * s2
        q[l + m, l - abs(m)] = 1j * (-1) ** m * s2
    q = (-1j) ** l * q
    dtype = {torch.float32: torch.complex64, torch.float64: torch.complex128}.get(dtype, torch.complex128)
    return q.to(dtype=dtype, device=device)


# --------------------------------------------------------------------------------------------
# Spherical harmonics (component normalisation, l <= 2)
# --------------------------------------------------------------------------------------------
def _spherical_harmonics(lmax, x, y, z):
    out = [torch.ones_like(x)]
    if lmax >= 1:
        s3 = math.sqrt(3.0)
        out += [s3 * x, s3 * y, s3 * z]
    if lmax >= 2:
        s5, s15 = math.sqrt(5.0), math.sqrt(15.0)
        out += [
            s15 * x * z,
            s15 * x * y,
            s5 * (y * y - 0.5 * (x * x + z * z)),
            s15 * y * z,
            0.5 * s15 * (z * z - x * x),
        ]
    if lmax > 2:
        raise NotImplementedError("shim spherical harmonics stop at l=2")
    return torch.stack(out, dim=-1)


def spherical_harmonics(l, x, normalize=True, normalization="component"):
    if isinstance(l, int):
        ls = [l]
    else:
        ls = list(l)
    if normalize:
        x = torch.nn.functional.normalize(x, dim=-1)
    sh = _spherical_harmonics(max(ls), x[..., 0], x[..., 1], x[..., 2])
    parts = [sh[..., i * i:(i + 1) * (i + 1)] for i in ls]
    out = torch.cat(parts, dim=-1)
    if normalization == "integral":
        scale = torch.cat([torch.full((2 * i + 1,), math.sqrt(2 * i + 1) / math.sqrt(4 * math.pi)) / math.sqrt(2 * i + 1) for i in ls])
        out = out * scale.to(out)
    return out


# --------------------------------------------------------------------------------------------
# normalize2mom (e3nn.math)
# --------------------------------------------------------------------------------------------
def _second_moment(f):
    z, w = np.polynomial.hermite_e.hermegauss(200)  # weight exp(-z^2/2)
    w = w / math.sqrt(2 * math.pi)
    zt = torch.tensor(z, dtype=torch.float64)
    with torch.no_grad():
        fz = f(zt).double().numpy()
    return float(np.sum(w * fz * fz))


class normalize2mom(torch.nn.Module):
    def __init__(self, f, dtype=None, device=None):
        super().__init__()
        self.f = f
        with torch.no_grad():
            cst = _second_moment(f) ** -0.5
        if abs(cst - 1) < 1e-4:
            self._is_id = True
            self.cst = 1.0
        else:
            self._is_id = False
            self.cst = cst

    def forward(self, x):
        if self._is_id:
            return self.f(x)
        return self.f(x).mul(self.cst)


# --------------------------------------------------------------------------------------------
# Registration
# --------------------------------------------------------------------------------------------
class _Dummy:
    def __init__(self, *a, **k):
        pass


def _compile_mode(mode):
    def deco(obj):
        return obj
    return deco


def _mod(name, **attrs):
    m = types.ModuleType(name)
    for k, v in attrs.items():
        setattr(m, k, v)
    sys.modules[name] = m
    return m


_INSTALLED = False


def install():
    """Register the stand-ins and mount the reference package; returns the e2former package path."""
    global _INSTALLED
    if _INSTALLED:
        return E2F_DIR
    if not os.path.isdir(E2F_DIR):
        raise RuntimeError(f"reference sources not found at {E2F_DIR!r}: set E2A_REFERENCE_ROOT to the "
                           "reference checkout (the directory holding src/molfm)")

    e3nn = _mod("e3nn")
    o3 = _mod("e3nn.o3", Irreps=Irreps, Irrep=Irrep, spherical_harmonics=spherical_harmonics,
              FromS2Grid=_Dummy, ToS2Grid=_Dummy, so3_generators=None, Linear=_Dummy,
              TensorProduct=_Dummy, FullyConnectedTensorProduct=_Dummy)
    wig = _mod("e3nn.o3._wigner", _su2_clebsch_gordan=_su2_clebsch_gordan,
               change_basis_real_to_complex=change_basis_real_to_complex)
    shm = _mod("e3nn.o3._spherical_harmonics", _spherical_harmonics=_spherical_harmonics)
    o3._wigner = wig
    o3._spherical_harmonics = shm
    tpm = _mod("e3nn.o3._tensor_product")
    _mod("e3nn.o3._tensor_product._codegen", _sum_tensors=None, codegen_tensor_product_left_right=None,
         codegen_tensor_product_right=None)
    _mod("e3nn.o3._tensor_product._instruction", Instruction=_Dummy)
    o3._tensor_product = tpm
    util = _mod("e3nn.util", prod=lambda xs: int(np.prod(list(xs))))
    jit = _mod("e3nn.util.jit", compile_mode=_compile_mode)
    cg = _mod("e3nn.util.codegen", CodeGenMixin=object)
    util.jit = jit
    util.codegen = cg
    math_m = _mod("e3nn.math", normalize2mom=normalize2mom)
    nn_m = _mod("e3nn.nn", Gate=_Dummy, Activation=_Dummy, FullyConnectedNet=_Dummy)
    e3nn.o3, e3nn.util, e3nn.math, e3nn.nn = o3, util, math_m, nn_m

    tc = _mod("torch_cluster", radius_graph=None)
    tg = _mod("torch_geometric")
    tgd = _mod("torch_geometric.data", Data=dict, Batch=dict)
    tg.data = tgd
    _mod("opt_einsum_fx", optimize_einsums_full=None)
    fa = _mod("faiss")
    fa.contrib = _mod("faiss.contrib")
    fa.contrib.torch_utils = _mod("faiss.contrib.torch_utils")

    if REF_SRC not in sys.path:
        sys.path.insert(0, REF_SRC)
    # Bare packages: do not execute the reference's package __init__ chains.
    for name, path in [
        ("molfm", os.path.join(REF_SRC, "molfm")),
        ("molfm.models", os.path.join(REF_SRC, "molfm", "models")),
        ("molfm.models.e2former", E2F_DIR),
        ("molfm.models.e2former.wigner6j", os.path.join(E2F_DIR, "wigner6j")),
        ("molfm.models.e2former.triton_dr", os.path.join(E2F_DIR, "triton_dr")),
        ("molfm.models.e2former.sp", os.path.join(E2F_DIR, "sp")),
    ]:
        p = types.ModuleType(name)
        p.__path__ = [path]
        sys.modules[name] = p
    _mod("molfm.models.e2former.maceblocks", NonLinearDipoleReadoutBlock=_Dummy)
    _mod("molfm.models.e2former.wigner6j.base_tensor_product", Simple_TensorProduct=_Dummy,
         Simple_TensorProduct_oTchannel=_Dummy, _sum_tensors=None, slices_basis=None)
    _mod("molfm.models.e2former.wigner6j.tensor_product", E2TensorProductArbitraryOrder=_Dummy,
         DepthWiseTensorProduct_reducesameorder=_Dummy, Simple_TensorProduct_oTchannel=_Dummy)
    _INSTALLED = True
    return E2F_DIR


def load_reference():
    """Install the shim and import the reference modules used on the attention path."""
    install()
    import importlib

    mods = {}
    for short, name in [
        ("mu", "molfm.models.e2former.module_utils"),
        ("so2tp", "molfm.models.e2former.wigner6j.so2_tensor_product"),
        ("e2f", "molfm.models.e2former.e2former"),
        ("qk", "molfm.models.e2former.triton_dr.triton_sparse_qk_autograd"),
    ]:
        mods[short] = importlib.import_module(name)
    # The reference has no torch branch for the edge-degree outer product; its own commented-out
    # torch code (e2former.py:742-749) is the stand-in used here.
    def _edge_degree_outer_torch(edge_sh, edge_fea, query_index, num_queries, metadata=None):
        edge_outer = edge_sh.unsqueeze(-1) * edge_fea.unsqueeze(1)
        out = torch.zeros((num_queries, edge_sh.shape[1], edge_fea.shape[-1]),
                          device=edge_outer.device, dtype=edge_outer.dtype)
        out.index_add_(0, query_index.to(torch.long), edge_outer)
        return out

    mods["e2f"].edge_degree_outer_triton = _edge_degree_outer_torch
    return mods
