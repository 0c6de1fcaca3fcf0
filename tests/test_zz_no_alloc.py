"""The allocation-free query-side backward against the workspace one, through the C ABI.

``e2a_attn_bwd_query_noalloc`` exists for callers that cannot allocate device memory when they run
the backward (an operator plugin that is handed only its tensors, code that must not call cudaMalloc
because it synchronises the device).  It keeps its scratch in a fixed array inside the library, so
this test checks that it gives the same results as ``e2a_attn_bwd_query`` with a caller workspace,
on two calls in a row (the array keeps the previous call's contents), and that sizes beyond the
array are refused.  This file is collected last on purpose.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(N=70, M=90, E=6000, H=128, D=8, C=58, seed=0):
    from ubio_molfm_b200 import _lib
    from ubio_molfm_b200._lib import check, ptr, stream_of
    from ubio_molfm_b200.ops import prepare_sparse_qk_edge_index_metadata

    dev = torch.device("cuda")
    rng = np.random.default_rng(seed)
    q_idx = torch.tensor(np.sort(rng.integers(0, N, E)), device=dev)
    n_idx = torch.tensor(rng.integers(0, M, E), device=dev)
    md = prepare_sparse_qk_edge_index_metadata(q_idx, n_idx, N, M)
    g = torch.Generator(device=dev).manual_seed(seed)
    t = {"q": torch.randn(N, H, D, device=dev, generator=g) / D ** 0.5,
         "k": torch.randn(M, H, D, device=dev, generator=g),
         "v": torch.randn(M, C, H, device=dev, generator=g),
         "gi": torch.randn(E, 2 * H, device=dev, generator=g),
         "poly": torch.rand(E, device=dev, generator=g),
         "dist": 1 + 4 * torch.rand(E, device=dev, generator=g),
         "dout": torch.randn(N, C, H, device=dev, generator=g)}
    lib = _lib.load()
    out = torch.empty(N, C, H, device=dev)
    beta = torch.empty(E, H, device=dev)
    rmax = torch.empty(N, H, device=dev)
    rsum = torch.empty(N, H, device=dev)
    st = stream_of(dev)
    check(lib.e2a_attn_fwd(ptr(t["q"]), ptr(t["k"]), ptr(t["v"]), ptr(t["gi"]), ptr(t["gi"][:, H:]), 2 * H,
                           ptr(t["poly"]), ptr(t["dist"]), ptr(md[0]), ptr(md[1]), None, N, M, E, H, D, C,
                           ptr(out), ptr(beta), ptr(rmax), ptr(rsum), st), "e2a_attn_fwd")
    return lib, md, t, beta, rmax, rsum, (N, M, E, H, D, C)


def _outputs(shape, dev="cuda"):
    N, M, E, H, D, C = shape
    return {"dq": torch.full((N, H, D), 7.0, device=dev), "dg": torch.full((E, 2 * H), 7.0, device=dev),
            "dp": torch.full((E,), 7.0, device=dev), "dd": torch.full((E,), 7.0, device=dev),
            "dl": torch.full((E, H), 7.0, device=dev)}


def _args(md, t, beta, rmax, rsum, shape, o):
    from ubio_molfm_b200._lib import ptr

    N, M, E, H, D, C = shape
    return [ptr(t["q"]), ptr(t["k"]), ptr(t["v"]), ptr(t["gi"]), ptr(t["gi"][:, H:]), 2 * H, ptr(t["poly"]),
            ptr(t["dist"]), ptr(md[0]), ptr(md[1]), None, N, M, E, H, D, C, ptr(beta), ptr(rmax), ptr(rsum),
            ptr(t["dout"]), ptr(o["dq"]), ptr(o["dg"]), ptr(o["dg"][:, H:]), 2 * H, ptr(o["dp"]), ptr(o["dd"]),
            ptr(o["dl"])]


def test_noalloc_backward_matches_workspace_backward_twice():
    from ubio_molfm_b200._lib import check, ptr, stream_of

    dev = torch.device("cuda")
    st = stream_of(dev)
    for seed in (0, 1):  # two calls in a row; the second sees the first call's leftovers in the array
        lib, md, t, beta, rmax, rsum, shape = _setup(seed=seed)
        E, H = shape[2], shape[3]
        ref = _outputs(shape)
        ws = torch.empty(lib.e2a_attn_bwd_workspace_bytes(E, H), dtype=torch.uint8, device=dev)
        check(lib.e2a_attn_bwd_query(*_args(md, t, beta, rmax, rsum, shape, ref), ptr(ws), ws.numel(), st),
              "e2a_attn_bwd_query")
        got = _outputs(shape)
        check(lib.e2a_attn_bwd_query_noalloc(*_args(md, t, beta, rmax, rsum, shape, got), st),
              "e2a_attn_bwd_query_noalloc")
        torch.cuda.synchronize()
        for key in ref:
            torch.testing.assert_close(got[key], ref[key], atol=1e-5, rtol=1e-5)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from ubio_molfm_b200 import _lib

    lib = _lib.load()
    # n_edges * H = 9000 * 128 > 2^20: refused before any launch (status 3, workspace too small)
    rc = lib.e2a_attn_bwd_query_noalloc(None, None, None, None, None, 256, None, None, None, None, None, 10, 10,
                                        9000, 128, 8, 58, None, None, None, None, None, None, None, 256, None, None,
                                        None, None)
    assert rc == 3


def test_noalloc_backward_matches_oracle_gradients():
    """The allocation-free entry point's gradients directly against the CPU oracle of the reference's
    attention span (float64 autograd), with the span parity tolerances (5e-5 of the largest gradient);
    every output starts filled with 7.0 so an element the kernel leaves unwritten shows."""
    import os
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import attention_ref as R
    from ubio_molfm_b200._lib import check, stream_of

    dev = torch.device("cuda")
    for seed in (2, 3):
        lib, md, t, beta, rmax, rsum, shape = _setup(seed=seed)
        N, M, E, H, D, C = shape
        got = _outputs(shape)
        check(lib.e2a_attn_bwd_query_noalloc(*_args(md, t, beta, rmax, rsum, shape, got), stream_of(dev)),
              "e2a_attn_bwd_query_noalloc")
        torch.cuda.synchronize()
        ins = [t[k].detach().cpu().double().requires_grad_(True) for k in ("q", "k", "v", "gi", "poly", "dist")]
        q_idx = torch.repeat_interleave(torch.arange(N), torch.diff(md[0].cpu().long()))
        n_idx = md[1].cpu().long()
        ref = R.attention_span(*ins, q_idx, n_idx, N)
        gq, _, _, ggi, gp, gd = torch.autograd.grad(ref, ins, t["dout"].cpu().double())
        for name, a, b in [("d_q", got["dq"], gq), ("d_gate/d_inputhead", got["dg"], ggi), ("d_poly", got["dp"], gp),
                           ("d_dist", got["dd"], gd)]:
            tol = 5e-5 * max(b.abs().max().item(), 1.0)
            assert (a.cpu().double() - b).abs().max().item() <= tol, name
