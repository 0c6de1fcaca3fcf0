"""ctypes binding of ``libe2a.so`` (the C ABI declared in ``include/e2a.h``).

The library is built in-tree (``python __graft_entry__.py`` / ``make -C ubio_molfm_b200/csrc``).
There is no fallback: if the library is missing or a call fails, the error is raised.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("E2A_LIB", os.path.join(_HERE, "libe2a.so"))

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
U64 = ctypes.c_uint64
F32 = ctypes.c_float
SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/e2a.h
SIGNATURES = {
    "e2a_version": (I32, []),
    "e2a_status_string": (ctypes.c_char_p, [I32]),
    "e2a_last_cuda_error": (I32, []),
    "e2a_launch_count": (U64, []),
    "e2a_csr_workspace_bytes": (SZ, [I64, I64, I64]),
    "e2a_csr_build": (I32, [P, P, I64, I64, I64, P, P, P, P, P, P, P, SZ, P]),
    "e2a_pbc_expand_workspace_bytes": (SZ, [I64, I32]),
    "e2a_pbc_expand": (I32, [P, I64, P, I32, F32, P, P, P, P, SZ, P]),
    "e2a_radius_graph_workspace_bytes": (SZ, [I64, I64, I64]),
    "e2a_radius_graph_plan": (I32, [P, P, P, P, I64, I64, I64, F32, F32, I64, P, P, P, SZ, P]),
    "e2a_radius_graph_fill_workspace_bytes": (SZ, [I64]),
    "e2a_radius_graph_fill": (I32, [P, P, P, P, I64, I64, I64, F32, F32, I64, I64, I64,
                                    P, P, P, P, P, P, P, P, SZ, P, SZ, P]),
    "e2a_sparse_qk_fwd": (I32, [P, P, P, P, P, I64, I64, I32, I32, P, P]),
    "e2a_grouped_reduce": (I32, [P, P, P, P, P, I64, I32, I32, P, P]),
    "e2a_alpha_sum_fwd": (I32, [P, P, P, I64, I32, P, P]),
    "e2a_alpha_sum_bwd": (I32, [P, P, I64, I32, P, P]),
    "e2a_v_agg_fwd": (I32, [P, P, P, P, P, I64, I32, I32, P, P]),
    "e2a_v_agg_fwd_bf16": (I32, [P, P, P, P, P, I64, I32, I32, P, P]),
    "e2a_v_agg_bwd_alpha": (I32, [P, P, P, P, P, I64, I32, I32, P, P]),
    "e2a_v_agg_bwd_value": (I32, [P, P, P, P, P, I64, I32, I32, P, P]),
    "e2a_edge_outer_fwd": (I32, [P, P, P, P, I64, I32, I32, P, P]),
    "e2a_edge_outer_bwd": (I32, [P, P, P, P, I64, I32, I32, P, P, P]),
    "e2a_attn_fwd": (I32, [P, P, P, P, P, I64, P, P, P, P, P, I64, I64, I64, I32, I32, I32,
                           P, P, P, P, P]),
    "e2a_attn_fwd_logits": (I32, [P, P, P, P, P, I64, P, P, P, P, P, I64, I64, I64, I32, I32, I32,
                                  P, P, P, P, P, P]),
    "e2a_attn_bwd_workspace_bytes": (SZ, [I64, I32]),
    "e2a_attn_bwd_query": (I32, [P, P, P, P, P, I64, P, P, P, P, P, I64, I64, I64, I32, I32, I32,
                                 P, P, P, P, P, P, P, I64, P, P, P, P, SZ, P]),
    "e2a_gemm_tf32x3": (I32, [P, I64, P, P, I64, P, I64, P, I64, I64, I64, I32, I32, P]),
    "e2a_tf32_split": (I32, [P, I64, I64, I64, P, P, I64, P]),
    "e2a_gemm_status": (I32, [P, I32, P]),
    "e2a_gemm_wait_selftest": (I32, [I64, P]),
    "e2a_gemm_tf32x3_pairprod": (I32, [P, I64, P, P, I64, P, I64, P, P, I64, I64, I64, I64, I32, I32, P]),
    "e2a_pair_grad": (I32, [P, P, I64, I32, I32, I32, P, P]),
    "e2a_gemm_tf32x3_pairgrad": (I32, [P, I64, P, I64, P, P, I64, P, I64, I64, I64, I64, I32, P]),
    "e2a_node_apply_fwd": (I32, [P, P, I64, P, I64, I64, I32, I32, I32, P, I64, I32, P]),
    "e2a_node_apply_bwd": (I32, [P, P, I64, P, I64, P, I64, I64, I32, I32, I32, P, I64, P, I64, P, P]),
    "e2a_rbf_fwd": (I32, [P, I64, P, I32, ctypes.c_float, P, P]),
    "e2a_gemm_tf32x3_rbf": (I32, [P, P, ctypes.c_float, P, P, I64, P, I64, P, I64, I64, I64, I32, P]),
    "e2a_gemm_tf32x3_rbf_dist_grad": (I32, [P, I64, P, P, I64, P, P, ctypes.c_float, P, I64, I64, I64, I64, I32, P]),
    "e2a_rbf_bwd": (I32, [P, P, I64, P, I32, ctypes.c_float, P, P]),
    "e2a_node_map_fwd": (I32, [P, I64, P, P, P, P, P, P, P]),
    "e2a_node_map_bwd": (I32, [P, P, I64, P, P, P, P, P, P, P]),
    "e2a_rms_norm_fwd": (I32, [P, I64, I32, I32, P, P, ctypes.c_float, P, P, P]),
    "e2a_rms_norm_bwd": (I32, [P, P, I64, I32, I32, P, P, P, P]),
    "e2a_gate_fwd": (I32, [P, P, I64, I32, I32, ctypes.c_float, ctypes.c_float, P, P]),
    "e2a_gate_bwd": (I32, [P, P, P, I64, I32, I32, ctypes.c_float, ctypes.c_float, P, P, P]),
    "e2a_ln_silu_fwd": (I32, [P, P, P, P, P, P, P, I64, I32, F32, P, P, P, P, P]),
    "e2a_ln_silu_bwd": (I32, [P, P, P, P, P, P, I64, I32, P, P]),
    "e2a_attn_bwd_query_noalloc": (I32, [P, P, P, P, P, I64, P, P, P, P, P, I64, I64, I64, I32, I32, I32,
                                         P, P, P, P, P, P, P, I64, P, P, P, P]),
    "e2a_attn_bwd_key": (I32, [P, P, P, P, P, P, P, P, I64, I64, I64, I32, I32, I32, P, P, P]),
    "e2a_attn_bwd_value": (I32, [P, P, P, P, P, P, P, I64, I64, I64, I32, I32, I32, P, P, P]),
    "e2a_attn_bwd_softmax_workspace_bytes": (SZ, [I64, I32]),
    "e2a_attn_bwd_softmax": (I32, [P, P, P, P, I64, P, P, P, P, P, I64, I64, I64, I32, I32, I32, P, P, P, P, P, P, P,
                                   I64, P, P, P, P, SZ, P]),
    "e2a_attn_bwd_softmax_logits": (I32, [P, P, P, I64, P, P, P, P, P, I64, I64, I64, I32, I32, I32, P, P, P, P, P,
                                          P, P, P, I64, P, P, P, P]),
    "e2a_attn_bwd_dk": (I32, [P, P, P, P, P, P, I64, I64, I64, I32, I32, I32, P, P]),
}

_lib = None


E2A_ERR_UNSUPPORTED = 4   # status of an entry point that does not take the given operands (include/e2a.h)


class E2AError(RuntimeError):
    pass


def load():
    """Load ``libe2a.so`` once and attach argument types; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise E2AError(f"libe2a.so not found at {LIB_PATH}: build it with `python __graft_entry__.py` "
                       "or `make -C ubio_molfm_b200/csrc` (there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def launch_count() -> int:
    """Kernels launched by this library so far in this process."""
    return int(load().e2a_launch_count())


def check(status: int, what: str):
    if status != 0:
        lib = load()
        msg = lib.e2a_status_string(status).decode()
        cuda = lib.e2a_last_cuda_error()
        raise E2AError(f"{what} failed: {msg} (status {status}, cudaError {cuda})")


def device_status_gemm(device=None, reset=True):
    """Status bits of the GEMM kernel's bounded waits (0 = nothing happened)."""
    lib = load()
    v = ctypes.c_uint(0)
    check(lib.e2a_gemm_status(ctypes.byref(v), 1 if reset else 0, stream_of(device)), "e2a_gemm_status")
    return int(v.value)


def raise_on_device_status(device=None):
    """Read and clear the GEMM's wait-status word; raise if a bounded wait gave up since the last check
    (the GEMM then left part of its output unwritten, so the results of that evaluation are invalid).
    One stream synchronisation."""
    st = device_status_gemm(device, reset=True)
    if st:
        raise E2AError(f"a tensor-core GEMM wait timed out on the device (status bits {st:#x}): the results "
                       "computed since the last check are invalid")


def gemm_wait_selftest(limit_ns=1_000_000, device=None):
    """Run one bounded wait that nothing completes (test hook): it gives up after ``limit_ns`` and sets
    the timeout bit that :func:`device_status_gemm` reports."""
    check(load().e2a_gemm_wait_selftest(int(limit_ns), stream_of(device)), "e2a_gemm_wait_selftest")


def ptr(t):
    """Device pointer of a tensor (None -> NULL)."""
    if t is None:
        return None
    return ctypes.c_void_p(t.data_ptr())


def stream_of(device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("ubio_molfm_b200 kernels need CUDA tensors (there is no CPU path)")
