"""Clebsch-Gordan selection tables for the first-order SO(2) tensor product (l2 = 1).

In each node's own frame the edge direction is the y axis, so the tensor product with the l=1
harmonic of r only touches its m=0 component (real index 1).  For every output (l3, m3) exactly one
input (l1, m1) has a non-zero coefficient; ``SO2_TP_givenl2`` (so2_tensor_product.py:182-271) stores
that input row as ``selected_idx`` and the coefficient as ``CG_weight``.

The coefficients are built from the standard Condon-Shortley SU(2) Clebsch-Gordan coefficients
(Racah's closed form) rotated to the real harmonic basis with e3nn's real<->complex change of basis
(including its ``(-i)^l`` phase), i.e. the same published construction the reference calls through
``e3nn.o3._wigner`` (so2_tensor_product.py:29-45).  Pure Python, float64, computed once at init.
"""
from __future__ import annotations

import math
from fractions import Fraction

import numpy as np


def _su2_cg(j1, m1, j2, m2, j3, m3):
    """<j1 m1 j2 m2 | j3 m3> for integer j (Racah formula, exact rational arithmetic)."""
    if m3 != m1 + m2 or not (abs(j1 - j2) <= j3 <= j1 + j2):
        return 0.0
    if abs(m1) > j1 or abs(m2) > j2 or abs(m3) > j3:
        return 0.0
    f = math.factorial
    pref = Fraction((2 * j3 + 1) * f(j3 + j1 - j2) * f(j3 - j1 + j2) * f(j1 + j2 - j3), f(j1 + j2 + j3 + 1))
    pref *= Fraction(f(j3 + m3) * f(j3 - m3) * f(j1 - m1) * f(j1 + m1) * f(j2 - m2) * f(j2 + m2), 1)
    s = Fraction(0)
    for k in range(0, j1 + j2 + j3 + 1):
        den = [k, j1 + j2 - j3 - k, j1 - m1 - k, j2 + m2 - k, j3 - j2 + m1 + k, j3 - j1 - m2 + k]
        if min(den) < 0:
            continue
        d = 1
        for x in den:
            d *= f(x)
        s += Fraction((-1) ** k, d)
    return float(s) * math.sqrt(float(pref))


def real_to_complex_basis(l):
    """e3nn's change of basis from real to complex harmonics of degree l, with the (-i)^l phase."""
    q = np.zeros((2 * l + 1, 2 * l + 1), dtype=np.complex128)
    r = 1.0 / math.sqrt(2.0)
    for m in range(-l, 0):
        q[l + m, l + abs(m)] = r
        q[l + m, l - abs(m)] = -1j * r
    q[l, l] = 1.0
    for m in range(1, l + 1):
        q[l + m, l + abs(m)] = (-1) ** m * r
        q[l + m, l - abs(m)] = 1j * (-1) ** m * r
    return ((-1j) ** l) * q


def real_cg(l1, l2, l3):
    """Real-basis coupling tensor C[m1, m2, m3] (unnormalised, as ``wigner_3j_wonorm(norm=False)``)."""
    C = np.zeros((2 * l1 + 1, 2 * l2 + 1, 2 * l3 + 1), dtype=np.complex128)
    for a, m1 in enumerate(range(-l1, l1 + 1)):
        for b, m2 in enumerate(range(-l2, l2 + 1)):
            for c, m3 in enumerate(range(-l3, l3 + 1)):
                C[a, b, c] = _su2_cg(l1, m1, l2, m2, l3, m3)
    Q1, Q2, Q3 = real_to_complex_basis(l1), real_to_complex_basis(l2), real_to_complex_basis(l3)
    R = np.einsum("ij,kl,mn,ikn->jlm", Q1, Q2, np.conj(Q3.T), C)
    if np.max(np.abs(R.imag)) > 1e-5:
        raise ValueError("real CG tensor has an imaginary part")
    return R.real


def so2_first_order_tables(lmax=2, l2=1):
    """Selection tables of the l2=1, l3 in [0, lmax] first-order SO(2) product.

    Returns ``(instructions, l3_sequential, selected_idx, cg_weight, path_norm)`` in the reference's
    ordering: instructions (l1, l3, start_l1) sorted by l3 (stable), output rows concatenated per
    instruction, ``l3_sequential = [[l3, count], ...]`` and ``path_norm`` = 1/sqrt(count) per row.
    """
    ins = []
    start = 0
    for l1 in range(lmax + 1):
        for l3 in range(abs(l1 - l2), l1 + l2 + 1):
            if l3 <= lmax:
                ins.append((l1, l3, start))
        start += 2 * l1 + 1
    ins = sorted(ins, key=lambda t: t[1])
    seq = []
    for _, l3, _ in ins:
        if seq and seq[-1][0] == l3:
            seq[-1][1] += 1
        else:
            seq.append([l3, 1])
    sel, w = [], []
    for l1, l3, s1 in ins:
        C = real_cg(l1, l2, l3)[:, l2]
        for m3 in range(2 * l3 + 1):
            nz = np.nonzero(C[:, m3])[0]
            if len(nz) == 0:
                sel.append(0)
                w.append(0.0)
            elif len(nz) == 1:
                sel.append(int(nz[0]) + s1)
                w.append(float(C[nz[0], m3]))
            else:
                raise ValueError("more than one coupled input component")
    norm = []
    for l3, cnt in seq:
        norm += [1.0 / math.sqrt(cnt)] * (2 * l3 + 1)
    return ins, seq, sel, w, norm
