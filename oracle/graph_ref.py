"""ctypes front-end of the C graph oracle (``graph_oracle.c``) -- TEST INFRASTRUCTURE ONLY.

Used by ``tests/`` and the bench's CPU-baseline leg to check / time the radius-graph path; see the
header of ``graph_oracle.c`` for the reference lines it restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def load():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liborc.so")
        if not os.path.exists(path):
            subprocess.check_call(["make", "-s", "-C", _HERE])
        lib = ctypes.CDLL(path)
        P = ctypes.c_void_p
        lib.orc_pbc_expand.restype = ctypes.c_int64
        lib.orc_pbc_expand.argtypes = [P, ctypes.c_int64, P, ctypes.c_int, ctypes.c_float, P]
        lib.orc_radius_graph.restype = ctypes.c_int64
        lib.orc_radius_graph.argtypes = [P, P, P, P, ctypes.c_int64, ctypes.c_float, ctypes.c_float, ctypes.c_int64,
                                         ctypes.c_int64, P, P, P]
        _LIB = lib
    return _LIB


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def pbc_expand(pos, offsets, cutoff):
    """-> image_atom (int64, c * n + a) of the kept images, in order."""
    pos = np.ascontiguousarray(pos, np.float32)
    off = np.ascontiguousarray(offsets, np.float32)
    n, nimg = pos.shape[0], off.shape[0]
    out = np.empty(n * nimg, np.int64)
    k = load().orc_pbc_expand(_p(pos), n, _p(off), nimg, float(cutoff), _p(out))
    return out[:k]


def radius_graph(pos, pts, q_ptr, p_ptr, max_dist, min_dist=-1.0, max_neighbors=None):
    """-> (query_idx, neighbor_idx, dist) with rows ordered by (distance, index)."""
    pos = np.ascontiguousarray(pos, np.float32)
    pts = np.ascontiguousarray(pts, np.float32)
    q_ptr = np.ascontiguousarray(q_ptr, np.int64)
    p_ptr = np.ascontiguousarray(p_ptr, np.int64)
    B = len(q_ptr) - 1
    mx = -1 if max_neighbors is None else int(max_neighbors)
    lib = load()
    cap = max(1, 64 * len(pos))
    while True:
        qi = np.empty(cap, np.int64)
        ni = np.empty(cap, np.int64)
        d = np.empty(cap, np.float32)
        E = lib.orc_radius_graph(_p(pos), _p(pts), _p(q_ptr), _p(p_ptr), B, float(max_dist), float(min_dist), mx,
                                 cap, _p(qi), _p(ni), _p(d))
        if E <= cap:
            return qi[:E], ni[:E], d[:E]
        cap = E
