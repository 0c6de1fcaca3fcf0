"""Per-node Wigner matrices of E2Former-V2 (module_utils.py:182-337, e2former.py:979-1015).

Each node's frame is the rotation taking its absolute position direction to the y axis:
beta = acos(y), alpha = atan2(x, z) (gamma = 0 at inference), and
``D^l = X(-gamma) J_l X(-beta) J_l X(-alpha)`` with ``X`` the rotation about y in the real
harmonic basis.  Computed in float64 on the device, cast to float32, as the reference does.
Entries at the poles / origin are detached exactly where the reference detaches them.

``J_l`` is the representation of the half-turn about (1,-1,0)/sqrt(2) (the rotation that exchanges
the x and -y axes); it is built here from the real spherical harmonics by a least-squares fit on
sample directions (float64, exact to ~1e-16), instead of being loaded from a data file.
"""
from __future__ import annotations

import math

import numpy as np
import torch


def _real_sh(l, v):
    x, y, z = v[..., 0], v[..., 1], v[..., 2]
    if l == 0:
        return np.ones(v.shape[:-1] + (1,))
    if l == 1:
        return math.sqrt(3.0) * np.stack([x, y, z], -1)
    if l == 2:
        s5, s15 = math.sqrt(5.0), math.sqrt(15.0)
        return np.stack([s15 * x * z, s15 * x * y, s5 * (y * y - 0.5 * (x * x + z * z)), s15 * y * z,
                         0.5 * s15 * (z * z - x * x)], -1)
    raise NotImplementedError("l <= 2")


def rotation_representation(l, R):
    """D^l(R) with Y_l(R v) = D^l(R) Y_l(v) in the component-normalised real basis (float64)."""
    V = np.random.default_rng(1234).normal(size=(64, 3))
    A, B = _real_sh(l, V), _real_sh(l, V @ np.asarray(R, np.float64).T)
    return np.linalg.lstsq(A, B, rcond=None)[0].T


_J_ROT = np.array([[0.0, -1.0, 0.0], [-1.0, 0.0, 0.0], [0.0, 0.0, 1.0]])


def jd_matrices(lmax=2):
    return [torch.tensor(rotation_representation(l, _J_ROT), dtype=torch.float64) for l in range(lmax + 1)]


def _y_rot(angle, l):
    """Rotation about y in the real basis of degree l: [..., 2l+1, 2l+1] (module_utils.py:275-302)."""
    M = angle.new_zeros(angle.shape + (2 * l + 1, 2 * l + 1))
    for i, f in enumerate(range(l, -l - 1, -1)):
        M[..., i, 2 * l - i] = torch.sin(f * angle)
        M[..., i, i] = torch.cos(f * angle)
    return M


def euler_angles(pos, eps=1e-5):
    """(alpha, beta, gamma) passed to the Wigner construction for node positions ``pos`` [N,3]
    (float64), i.e. the negated (gamma, beta, alpha) of module_utils.py:182-226 with gamma = 0."""
    d = torch.norm(pos, dim=1)
    small = d < eps
    d = torch.where(small, torch.ones_like(d), d)
    xyz = pos / d.view(-1, 1)
    y = xyz[:, 1]
    mask = small | torch.isclose(y.abs(), torch.ones_like(y))
    y_safe = torch.where(mask, torch.zeros_like(y), y)
    beta = torch.where(mask, torch.acos(y).detach(), torch.acos(y_safe))
    x_s = torch.where(mask, torch.ones_like(y), xyz[:, 0])
    z_s = torch.where(mask, torch.ones_like(y), xyz[:, 2])
    alpha = torch.where(mask, torch.atan2(xyz[:, 0], xyz[:, 2]).detach(), torch.atan2(x_s, z_s))
    gamma = torch.zeros_like(alpha)
    return -gamma, -beta, -alpha


def node_wigner(pos, lmax=2, l3_sequential=((0, 1), (1, 3), (2, 2)), dtype=torch.float32, jd=None):
    """``(wigner [N,(lmax+1)^2,(lmax+1)^2], wigner_inv [N,S,S])`` for node positions ``pos``.

    ``wigner_inv`` repeats the degree-l3 block ``count`` times per ``l3_sequential`` and is
    transposed (module_utils.py:305-337)."""
    p = pos.to(torch.float64)
    a, b, c = euler_angles(p)
    jd = jd_matrices(lmax) if jd is None else jd
    jd = [j.to(p.device) for j in jd]
    blocks = []
    for l in range(lmax + 1):
        J = jd[l]
        blocks.append(_y_rot(a, l) @ J @ _y_rot(b, l) @ J @ _y_rot(c, l))
    n = p.shape[0]
    size = (lmax + 1) ** 2
    W = p.new_zeros((n, size, size))
    s = 0
    for blk in blocks:
        k = blk.shape[-1]
        W[:, s:s + k, s:s + k] = blk
        s += k
    S = sum((2 * l + 1) * cnt for l, cnt in l3_sequential)
    Wi = p.new_zeros((n, S, S))
    s = 0
    for l, cnt in l3_sequential:
        for _ in range(cnt):
            k = 2 * l + 1
            Wi[:, s:s + k, s:s + k] = blocks[l]
            s += k
    return W.to(dtype), Wi.transpose(1, 2).contiguous().to(dtype)
