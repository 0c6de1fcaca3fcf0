"""Tensor-core fp32 projections: ``y = x W^T (+ b)`` on tcgen05 through ``e2a_gemm_tf32x3``.

The 3xTF32 split keeps fp32-level accuracy (parity mode); ``passes=1`` is plain TF32.  Only the
input gradient is produced by the CUDA path (what force evaluation needs); a weight gradient, when a
caller asks for one, is formed with ``torch.matmul``.
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, stream_of

PASSES = 3
# Pre-split the weight operand (B) into tf32 hi / lo once per call (one small launch) instead of
# splitting it on chip in every tile.
PRESPLIT_WEIGHTS = True


def first_order_only(name):
    """Raise for a second-order (``create_graph=True``) backward through an inference-only fused op: these
    treat their parameters as constants and have no differentiable backward.  Force-loss training runs the
    model in training mode, whose ops all have one."""
    raise RuntimeError(f"{name}: double backward (create_graph=True) is not supported by this eval-mode fused op; "
                       "put the model in training mode (model.train()) for force-loss training")


def split_tf32(b):
    """``b`` (fp32, rows of K) -> (hi, lo) contiguous with hi = tf32(b), lo = tf32(b - hi): the
    pre-split weight operand of the GEMM (one small launch, reused by every product with ``b`` or a
    row block of it)."""
    lib = _lib.load()
    b = b.contiguous().float()
    hi = torch.empty_like(b)
    lo = torch.empty_like(b)
    K = b.shape[-1]
    check(lib.e2a_tf32_split(ptr(b), K, b.numel() // max(K, 1), K, ptr(hi), ptr(lo), K, stream_of(b.device)),
          "e2a_tf32_split")
    return hi, lo


def _maybe_split(b):
    """``split_tf32(b)`` when weights are pre-split, else ``(b, None)`` (split on chip)."""
    return split_tf32(b) if PRESPLIT_WEIGHTS else (b.contiguous(), None)


def _presplit_ok(a_ptr, lda, K):
    return PRESPLIT_WEIGHTS and K > 0 and K % 4 == 0 and a_ptr % 16 == 0 and lda % 4 == 0


class GemmTimer:
    """Opt-in CUDA-event bracketing of every tensor-core GEMM launch with its product count (2MNK):
    used by the benchmark to report the projections' delivered TFLOP/s inside the model step."""

    def __init__(self):
        self.enabled = False
        self.records = []

    def start(self):
        if not self.enabled:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def stop(self, e0, M, N, K):
        if e0 is None:
            return
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record()
        self.records.append((e0, e1, 2.0 * M * N * K, (int(M), int(N), int(K))))

    def summary(self):
        """(launches, total ms, total flop); call after synchronising."""
        return (len(self.records), sum(r[0].elapsed_time(r[1]) for r in self.records),
                sum(r[2] for r in self.records))

    def by_shape(self, top=12):
        """[(M, N, K, launches, ms, TFLOP/s)] of the shapes that took the most time."""
        agg = {}
        for a, b, f, shp in self.records:
            o = agg.setdefault(shp, [0, 0.0, 0.0])
            o[0] += 1
            o[1] += a.elapsed_time(b)
            o[2] += f
        rows = sorted(agg.items(), key=lambda kv: -kv[1][1])[:top]
        return [(m, n, k, c, round(ms, 3), round(fl / ms / 1e9, 1)) for (m, n, k), (c, ms, fl) in rows]


GEMM_TIMER = GemmTimer()


def _gemm_ptrs(lib, a, lda, b, b_lo, ldb, c, ldc, bias, M, N, K, accumulate, passes, dev, P=None, ldp=0):
    """Raw-pointer GEMM (pair-product epilogue when ``P`` is given; ``b_lo`` = pre-split low part)."""
    t0 = GEMM_TIMER.start()
    try:
        _gemm_ptrs_launch(lib, a, lda, b, b_lo, ldb, c, ldc, bias, M, N, K, accumulate, passes, dev, P, ldp)
    finally:
        GEMM_TIMER.stop(t0, M, N, K)


def _gemm_ptrs_launch(lib, a, lda, b, b_lo, ldb, c, ldc, bias, M, N, K, accumulate, passes, dev, P=None, ldp=0):
    st = stream_of(dev)
    if P is not None:
        check(lib.e2a_gemm_tf32x3_pairprod(a, lda, b, b_lo, ldb, c, ldc, bias, P, ldp, M, N, K,
                                           1 if accumulate else 0, passes, st), "e2a_gemm_tf32x3_pairprod")
        return
    check(lib.e2a_gemm_tf32x3(a, lda, b, b_lo, ldb, c, ldc, bias, M, N, K, 1 if accumulate else 0, passes, st),
          "e2a_gemm_tf32x3")


def gemm(a, b, bias=None, out=None, accumulate=False, passes=None, b_split=None):
    """``a [M,K] @ b[N,K]^T (+ bias)`` -> [M,N] (fp32, CUDA, row-major with unit inner stride).
    ``b_split`` = rows of ``split_tf32`` output matching ``b`` when the caller reuses ``b``; with
    aligned operands ``b`` is split here otherwise."""
    lib = _lib.load()
    if a.dtype != torch.float32 or b.dtype != torch.float32:
        raise TypeError("gemm expects float32 operands")
    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[1]:
        raise ValueError(f"gemm shape mismatch {tuple(a.shape)} x {tuple(b.shape)}^T")
    if a.stride(1) != 1:
        a = a.contiguous()
    if b.stride(1) != 1:
        b = b.contiguous()
    M, K = a.shape
    N = b.shape[0]
    if out is None:
        out = torch.empty((M, N), device=a.device, dtype=torch.float32)
    if bias is not None:
        bias = bias.contiguous()
    lda = max(a.stride(0), K)
    passes = PASSES if passes is None else passes
    if _presplit_ok(a.data_ptr(), lda, K):
        hi, lo = b_split if b_split is not None else split_tf32(b)
        _gemm_ptrs(lib, ptr(a), lda, ptr(hi), ptr(lo), K, ptr(out), out.stride(0), ptr(bias), M, N, K, accumulate,
                   passes, a.device)
    else:
        _gemm_ptrs(lib, ptr(a), lda, ptr(b), None, max(b.stride(0), K), ptr(out), out.stride(0), ptr(bias), M, N, K,
                   accumulate, passes, a.device)
    return out


class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        y = gemm(x2, w, b)
        ctx.save_for_backward(x if w.requires_grad else None, w)
        ctx.shape = shape
        ctx.has_b = b is not None
        return y.reshape(*shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        x2 = None if x is None else x.reshape(-1, x.shape[-1])
        g2 = gy.reshape(-1, gy.shape[-1]).contiguous()
        dx = dw = db = None
        if torch.is_grad_enabled():
            # create_graph=True: dx through this same tensor-core op (differentiable in g and w), dw / db
            # as PyTorch products, so the gradients carry their own graph for force-loss training
            if ctx.needs_input_grad[0]:
                dx = _LinearFn.apply(g2, w.t(), None).reshape(ctx.shape)
            if ctx.needs_input_grad[1]:
                dw = g2.t() @ x2
            if ctx.has_b and ctx.needs_input_grad[2]:
                db = g2.sum(0)
            return dx, dw, db
        if ctx.needs_input_grad[0]:
            dx = gemm(g2, w.t().contiguous()).reshape(ctx.shape)
        if ctx.needs_input_grad[1]:
            dw = g2.t() @ x2
        if ctx.has_b and ctx.needs_input_grad[2]:
            db = g2.sum(0)
        return dx, dw, db


def linear(x, w, b=None):
    """``torch.nn.functional.linear`` on the tensor cores (CUDA fp32 inputs)."""
    if not x.is_cuda:
        raise ValueError("ubio_molfm_b200 kernels need CUDA tensors (there is no CPU path)")
    return _LinearFn.apply(x.float(), w, b)


class _SO3LinearFn(torch.autograd.Function):
    """``out[:, m, :] = x[:, m, :] @ W[l(m)]^T`` (+ bias on row 0) as one strided GEMM per row m.

    ``x`` is [N, R, C] contiguous; every row m is read in place as an [N, C] matrix with leading
    dimension R*C and written in place into ``out`` [N, R, C_out] -- no copies."""

    @staticmethod
    def forward(ctx, x, w, bias, lidx):
        N, R, C = x.shape
        Co = w.shape[1]
        x_in = x
        x = x.contiguous()
        out = torch.empty((N, R, Co), device=x.device, dtype=torch.float32)
        whi, wlo = _maybe_split(w)
        for m in range(R):
            gemm(x[:, m, :], w[lidx[m]], bias if (m == 0 and bias is not None) else None, out=out[:, m, :],
                 b_split=(whi[lidx[m]], wlo[lidx[m]]))
        ctx.save_for_backward(x_in if w.requires_grad else None, w)
        ctx.lidx = lidx
        ctx.has_bias = bias is not None
        return out

    @staticmethod
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        g = g.contiguous()
        N, R, Co = g.shape
        C = w.shape[2]
        dx = dw = db = None
        if torch.is_grad_enabled():
            # create_graph=True: the same strided op with W^T for dx, PyTorch products for dW
            if ctx.needs_input_grad[0]:
                dx = _SO3LinearFn.apply(g, w.transpose(1, 2).contiguous(), None, ctx.lidx)
            if ctx.needs_input_grad[1]:
                x = x.float()
                dw = torch.stack([sum(g[:, m, :].t() @ x[:, m, :] for m in range(R) if ctx.lidx[m] == l)
                                  if l in ctx.lidx else torch.zeros_like(w[l]) for l in range(w.shape[0])])
            if ctx.has_bias and ctx.needs_input_grad[2]:
                db = g[:, 0, :].sum(0)
            return dx, dw, db, None
        if ctx.needs_input_grad[0]:
            wt = w.transpose(1, 2).contiguous()  # [L, C, Co]
            thi, tlo = _maybe_split(wt)
            dx = torch.empty((N, R, C), device=g.device, dtype=torch.float32)
            for m in range(R):
                gemm(g[:, m, :], wt[ctx.lidx[m]], None, out=dx[:, m, :], b_split=(thi[ctx.lidx[m]], tlo[ctx.lidx[m]]))
        if ctx.needs_input_grad[1]:
            dw = torch.zeros_like(w)
            for m in range(R):
                dw[ctx.lidx[m]] += g[:, m, :].t() @ x[:, m, :]
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = g[:, 0, :].sum(0)
        return dx, dw, db, None


def so3_linear(x, w, bias, lidx):
    """Per-degree linear of [N, R, C] irreps features with weights [L+1, C_out, C] (CUDA)."""
    if not x.is_cuda:
        raise ValueError("ubio_molfm_b200 kernels need CUDA tensors (there is no CPU path)")
    return _SO3LinearFn.apply(x.float(), w, bias, tuple(int(v) for v in lidx))


class _LnSiluFn(torch.autograd.Function):
    """y = SiLU(LayerNorm(h [+ T[zt] + S[zs]])) with constant gamma / beta / tables (eval mode)."""

    @staticmethod
    def forward(ctx, h, gamma, beta, eps, T, zt, S, zs):
        lib = _lib.load()
        h = h.contiguous()
        rows, W = h.shape
        y = torch.empty_like(h)
        mean = torch.empty(rows, device=h.device, dtype=torch.float32)
        rstd = torch.empty_like(mean)
        x = torch.empty_like(h) if T is not None else h
        check(lib.e2a_ln_silu_fwd(ptr(h), ptr(T), ptr(zt), ptr(S), ptr(zs), ptr(gamma), ptr(beta), rows, W, float(eps),
                                  ptr(x) if T is not None else None, ptr(y), ptr(mean), ptr(rstd),
                                  stream_of(h.device)), "e2a_ln_silu_fwd")
        ctx.save_for_backward(x, gamma, beta, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        if torch.is_grad_enabled():
            first_order_only("ln_silu")
        lib = _lib.load()
        x, gamma, beta, mean, rstd = ctx.saved_tensors
        dy = dy.contiguous()
        dx = torch.empty_like(dy)
        rows, W = dy.shape
        check(lib.e2a_ln_silu_bwd(ptr(x), ptr(dy), ptr(gamma), ptr(beta), ptr(mean), ptr(rstd), rows, W, ptr(dx),
                                  stream_of(dy.device)), "e2a_ln_silu_bwd")
        return dx, None, None, None, None, None, None, None


def ln_silu_supported(W):
    return W % 128 == 0 and W <= 1024


def ln_silu(h, ln, tables=None):
    """Fused SiLU(LayerNorm(h + tables)) for a 2-D CUDA tensor, LayerNorm module ``ln`` (constants).

    ``tables`` = (T, zt, S, zs): per-row gathered table rows T[zt] + S[zs] added before the norm."""
    T = zt = S = zs = None
    if tables is not None:
        T, zt, S, zs = (t.contiguous() for t in tables)
    return _LnSiluFn.apply(h.float(), ln.weight.detach().contiguous(), ln.bias.detach().contiguous(), ln.eps,
                           T, zt, S, zs)


# Backward of the pair product: True = D = pair_grad(O, G) formed inside the GEMM's A tiles
# (e2a_gemm_tf32x3_pairgrad; D never reaches HBM), False = pair_grad kernel then the plain GEMM.
FUSED_PAIR_GRAD = True


class _SO3PairProdFn(torch.autograd.Function):
    """``P[n, l, j] = sum_{m in degree l} o1[n,m,j] * o2[n,m,j]`` with ``o1 = x W1[l]^T (+b on m=0)``,
    ``o2 = x W2[l]^T`` (the inner product of SO3_Linear2Scalar_e2former), fused into the GEMM
    epilogue.  ``w12`` [L+1, 2h, C] holds W1 / W2 rows interleaved; ``b12`` [2h] the bias (0 on odd).
    With ``recompute`` the projections O are not kept for the backward (they are 4h floats per row,
    the largest per-node activation of the layer) but formed again there from ``x`` by the same GEMMs,
    so the backward sees the same values."""

    @staticmethod
    def _project(lib, x, whi, wlo, b12, lidx, O, P=None):
        N, R, C = x.shape
        L1, h2 = whi.shape[0], whi.shape[1]
        dev = x.device
        for m in range(R):
            l = lidx[m]
            first = m == l * l
            _gemm_ptrs(lib, x[:, m, :].data_ptr(), R * C, ptr(whi[l]), ptr(wlo[l]) if wlo is not None else None, C,
                       ptr(O[:, m, :]), R * h2, ptr(b12) if m == 0 else None, N, h2, C,
                       P is not None and not first, PASSES, dev,
                       P=ptr(P[:, l, :]) if P is not None else None, ldp=L1 * (h2 // 2))

    @staticmethod
    def forward(ctx, x, w12, b12, lidx, recompute=False):
        lib = _lib.load()
        x = x.contiguous()
        N, R, C = x.shape
        L1, h2, _ = w12.shape
        h = h2 // 2
        dev = x.device
        O = torch.empty((N, R, h2), device=dev, dtype=torch.float32)
        P = torch.empty((N, L1, h), device=dev, dtype=torch.float32)
        whi, wlo = split_tf32(w12) if _presplit_ok(x.data_ptr(), R * C, C) else (w12, None)
        _SO3PairProdFn._project(lib, x, whi, wlo, b12, lidx, O, P)
        if recompute:
            del O
            ctx.save_for_backward(x, w12, b12)
        else:
            ctx.save_for_backward(O, w12, b12)
        ctx.recompute = recompute
        ctx.lidx = lidx
        return P

    @staticmethod
    def backward(ctx, G):
        if torch.is_grad_enabled():
            first_order_only("so3_pair_product")
        lib = _lib.load()
        t0, w12, b12 = ctx.saved_tensors
        if ctx.recompute:
            x = t0
            O = torch.empty((x.shape[0], x.shape[1], w12.shape[1]), device=x.device, dtype=torch.float32)
            whi, wlo = split_tf32(w12) if _presplit_ok(x.data_ptr(), x.shape[1] * x.shape[2], x.shape[2]) else (w12, None)
            _SO3PairProdFn._project(lib, x, whi, wlo, b12, ctx.lidx, O)
        else:
            O = t0
        G = G.contiguous()
        N, R, h2 = O.shape
        L1 = w12.shape[0]
        C = w12.shape[2]
        wt = w12.transpose(1, 2).contiguous()  # [L+1, C, 2h]
        thi, tlo = _maybe_split(wt)
        dx = torch.empty((N, R, C), device=O.device, dtype=torch.float32)
        if FUSED_PAIR_GRAD and tlo is not None and h2 % 32 == 0 and O.data_ptr() % 16 == 0 and G.data_ptr() % 16 == 0:
            # D = pair_grad(O, G) formed inside the GEMM's A tiles, one launch per irreps row (rows whose
            # operands the fused kernel does not take report E2A_ERR_UNSUPPORTED before any launch and
            # go the two-kernel way below)
            st = stream_of(O.device)
            done = True
            for m in range(R):
                l = ctx.lidx[m]
                t0 = GEMM_TIMER.start()
                rc = lib.e2a_gemm_tf32x3_pairgrad(O.data_ptr() + 4 * m * h2, R * h2, G.data_ptr() + 4 * l * (h2 // 2),
                                                  L1 * (h2 // 2), ptr(thi[l]), ptr(tlo[l]), h2,
                                                  dx.data_ptr() + 4 * m * C, R * C, N, C, h2, PASSES, st)
                if rc == _lib.E2A_ERR_UNSUPPORTED and m == 0:
                    done = False
                    break
                check(rc, "e2a_gemm_tf32x3_pairgrad")
                GEMM_TIMER.stop(t0, N, C, h2)
            if done:
                return dx, None, None, None, None
        D = torch.empty_like(O)
        check(lib.e2a_pair_grad(ptr(O), ptr(G), N, R, L1, h2 // 2, ptr(D), stream_of(O.device)), "e2a_pair_grad")
        for m in range(R):
            gemm(D[:, m, :], wt[ctx.lidx[m]], None, out=dx[:, m, :], b_split=(thi[ctx.lidx[m]], tlo[ctx.lidx[m]]))
        return dx, None, None, None, None


def so3_pair_product(x, w1, w2, bias, lidx, recompute=False):
    """Fused per-degree inner product of two per-degree linears (constant weights)."""
    if not x.is_cuda:
        raise ValueError("ubio_molfm_b200 kernels need CUDA tensors (there is no CPU path)")
    L1, h, C = w1.shape
    w12 = torch.stack([w1, w2], dim=2).reshape(L1, 2 * h, C).contiguous()
    b12 = torch.stack([bias.reshape(-1), torch.zeros_like(bias.reshape(-1))], dim=1).reshape(2 * h).contiguous()
    return _SO3PairProdFn.apply(x.float(), w12, b12, tuple(int(v) for v in lidx), bool(recompute))


class _NodeApplyFn(torch.autograd.Function):
    """Per-node [20 x 9] map of irreps rows, A [n, 20, 9]:

    * ``plain``: out [n, 20, C] = A h for h [n, 9, C] (h may be a row-strided view);
    * ``merge``: out [n, 29, C] = [A h ; h]  (the value rows appended after the product rows);
    * ``sub``:   out [n, 20, C] = A x[:, 20:] - x[:, :20] for x [n, 29, C]  (gradient w.r.t. x).
    """

    @staticmethod
    def forward(ctx, A, h, mode):
        lib = _lib.load()
        A_in, h_in = A, h
        A = A.contiguous()
        n, KO, KI = A.shape
        C = h.shape[2]
        if h.stride(2) != 1 or h.stride(1) != C:
            h = h.contiguous()
        dev = h.device
        if mode == "sub":
            src, sub = h[:, KO:], h
            out = torch.empty((n, KO, C), device=dev, dtype=torch.float32)
            check(lib.e2a_node_apply_fwd(ptr(A), ptr(src), h.stride(0), ptr(sub), h.stride(0), n, KO, KI, C, ptr(out),
                                         out.stride(0), 0, stream_of(dev)), "e2a_node_apply_fwd")
            h = src.contiguous()   # the backward reads only the value rows; keep [n, 9, C], not all 29
        else:
            rows = KO + KI if mode == "merge" else KO
            out = torch.empty((n, rows, C), device=dev, dtype=torch.float32)
            check(lib.e2a_node_apply_fwd(ptr(A), ptr(h), h.stride(0), None, 0, n, KO, KI, C, ptr(out), out.stride(0),
                                         1 if mode == "merge" else 0, stream_of(dev)), "e2a_node_apply_fwd")
            h = h_in
        ctx.save_for_backward(A_in, h)
        ctx.mode = mode
        return out

    @staticmethod
    def backward(ctx, g):
        lib = _lib.load()
        A, h = ctx.saved_tensors
        if torch.is_grad_enabled():
            # create_graph=True: the bilinear map's gradients as batched products that carry their own graph
            if ctx.mode == "sub":
                first_order_only("node_apply(mode='sub')")
            KO = A.shape[1]
            gp = g[:, :KO]
            dA = torch.bmm(gp, h.transpose(1, 2)) if ctx.needs_input_grad[0] else None
            dh = None
            if ctx.needs_input_grad[1]:
                dh = torch.bmm(A.transpose(1, 2), gp)
                if ctx.mode == "merge":
                    dh = dh + g[:, KO:]
            return dA, dh, None
        A = A.contiguous()
        if h.stride(2) != 1 or h.stride(1) != h.shape[2]:
            h = h.contiguous()
        g = g.contiguous()
        n, KO, KI = A.shape
        C = h.shape[2]
        dev = h.device
        dA = torch.empty_like(A) if ctx.needs_input_grad[0] else None
        if ctx.mode == "sub":
            dx = torch.empty((n, KO + KI, C), device=dev, dtype=torch.float32)
            check(lib.e2a_node_apply_bwd(ptr(A), ptr(h), h.stride(0), ptr(g), g.stride(0), None, 0, n, KO, KI,
                                         C, ptr(dx[:, KO:]), dx.stride(0), ptr(dx), dx.stride(0), ptr(dA),
                                         stream_of(dev)), "e2a_node_apply_bwd")
            return dA, dx, None
        dh = torch.empty((n, KI, C), device=dev, dtype=torch.float32)
        add = g[:, KO:] if ctx.mode == "merge" else None
        check(lib.e2a_node_apply_bwd(ptr(A), ptr(h), h.stride(0), ptr(g), g.stride(0), ptr(add),
                                     g.stride(0) if add is not None else 0, n, KO, KI, C, ptr(dh), dh.stride(0),
                                     None, 0, ptr(dA), stream_of(dev)), "e2a_node_apply_bwd")
        return dA, dh, None


def node_apply(A, h, mode="plain"):
    """Per-node [20 x 9] map of irreps rows (CUDA); ``mode`` as in :class:`_NodeApplyFn`."""
    if mode not in ("plain", "merge", "sub"):
        raise ValueError(f"unknown node_apply mode {mode!r}")
    return _NodeApplyFn.apply(A.float(), h.float(), mode)


class _RowBlockLinearFn(torch.autograd.Function):
    """out[n, o_t, :] = x[n, r_t : r_t + k_t, :].flatten() @ W_t^T (+ bias on output row 0), one
    tensor-core GEMM per task t = (r_t, k_t, o_t, w_t) with node-strided operands (no copies).  The
    tasks partition the rows of x, so the input gradient is written, not accumulated.  Weights are
    constants (inference path)."""

    @staticmethod
    def forward(ctx, x, tasks, weights, weights_t, bias, out_rows):
        lib = _lib.load()
        x = x.contiguous()
        n, R, C = x.shape
        Co = weights[0].shape[0]
        out = torch.empty((n, out_rows, Co), device=x.device, dtype=torch.float32)
        splits = [_maybe_split(w) for w in weights]
        for r0, k, o, wi in tasks:
            _gemm_ptrs(lib, x.data_ptr() + 4 * r0 * C, R * C, ptr(splits[wi][0]), ptr(splits[wi][1]), k * C,
                       out.data_ptr() + 4 * o * Co, out_rows * Co, ptr(bias) if (bias is not None and o == 0) else None,
                       n, Co, k * C, False, PASSES, x.device)
        ctx.tasks, ctx.weights_t, ctx.shape = tasks, weights_t, (n, R, C, out_rows, Co)
        return out

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            first_order_only("rowblock_linear")
        lib = _lib.load()
        g = g.contiguous()
        n, R, C, out_rows, Co = ctx.shape
        dx = torch.empty((n, R, C), device=g.device, dtype=torch.float32)
        splits = [_maybe_split(w) for w in ctx.weights_t]
        for r0, k, o, wi in ctx.tasks:
            _gemm_ptrs(lib, g.data_ptr() + 4 * o * Co, out_rows * Co, ptr(splits[wi][0]), ptr(splits[wi][1]), Co,
                       dx.data_ptr() + 4 * r0 * C, R * C, None, n, k * C, Co, False, PASSES, g.device)
        return dx, None, None, None, None, None


def rowblock_linear(x, tasks, weights, bias, out_rows):
    """See :class:`_RowBlockLinearFn`; ``weights`` are [Co, k*C] fp32 CUDA tensors."""
    rows = sorted((r0, r0 + k) for r0, k, _, _ in tasks)
    if rows[0][0] != 0 or rows[-1][1] != x.shape[1] or any(a[1] != b[0] for a, b in zip(rows, rows[1:])):
        raise ValueError("rowblock_linear tasks must partition the input rows")
    weights = [w.detach().float().contiguous() for w in weights]
    weights_t = [w.t().contiguous() for w in weights]
    b = bias.detach().float().contiguous() if bias is not None else None
    return _RowBlockLinearFn.apply(x.float(), tuple(tasks), weights, weights_t, b, out_rows)


# ------------------------------------------------------------------------------------------------
# Node-wise block kernels: equivariant RMS norm and the gated activation (inference path)
# ------------------------------------------------------------------------------------------------
def rms_norm_supported(x):
    return x.is_cuda and x.dim() == 3 and x.shape[1] in (1, 4, 9) and x.shape[2] in (128, 256)


class _RmsNormFn(torch.autograd.Function):
    """EquivariantRMSNormArraySphericalHarmonicsV2_BL with constant affine parameters."""

    @staticmethod
    def forward(ctx, x, w, b, eps):
        lib = _lib.load()
        x = x.contiguous()
        n, R, C = x.shape
        y = torch.empty_like(x)
        stats = torch.empty((n, 2), device=x.device, dtype=torch.float32)
        check(lib.e2a_rms_norm_fwd(ptr(x), n, R, C, ptr(w), ptr(b), float(eps), ptr(y), ptr(stats),
                                   stream_of(x.device)), "e2a_rms_norm_fwd")
        ctx.save_for_backward(x, w, stats)
        return y

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            first_order_only("rms_norm")
        lib = _lib.load()
        x, w, stats = ctx.saved_tensors
        g = g.contiguous()
        n, R, C = x.shape
        dx = torch.empty_like(x)
        check(lib.e2a_rms_norm_bwd(ptr(x), ptr(g), n, R, C, ptr(w), ptr(stats), ptr(dx), stream_of(x.device)),
              "e2a_rms_norm_bwd")
        return dx, None, None, None


def rms_norm(x, weight, bias, eps):
    """Equivariant RMS norm of [n, (lmax+1)^2, C] irreps (CUDA; constant weight [lmax+1, C], bias [C])."""
    return _RmsNormFn.apply(x.float(), weight.detach().float().contiguous(), bias.detach().float().contiguous(),
                            float(eps))


class _GateFn(torch.autograd.Function):
    """Gate_s3: y[0] = cs silu(s[0]), y[r] = cv sigmoid(s[l(r)]) h[r]."""

    @staticmethod
    def forward(ctx, s, h, cs, cv):
        lib = _lib.load()
        s = s.contiguous()
        h = h.contiguous()
        n, R, C = h.shape
        y = torch.empty_like(h)
        check(lib.e2a_gate_fwd(ptr(s), ptr(h), n, R, C, float(cs), float(cv), ptr(y), stream_of(h.device)),
              "e2a_gate_fwd")
        ctx.save_for_backward(s, h)
        ctx.c = (float(cs), float(cv))
        return y

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            first_order_only("gate")
        lib = _lib.load()
        s, h = ctx.saved_tensors
        g = g.contiguous()
        n, R, C = h.shape
        ds = torch.empty_like(s)
        dh = torch.empty_like(h)
        check(lib.e2a_gate_bwd(ptr(s), ptr(h), ptr(g), n, R, C, ctx.c[0], ctx.c[1], ptr(ds), ptr(dh),
                               stream_of(h.device)), "e2a_gate_bwd")
        return ds, dh, None, None


def gate(s, h, c_scalar, c_vector):
    """Gated activation of irreps rows ``h`` [n, 9, C] by gate pre-activations ``s`` [n, 3 C] (CUDA)."""
    return _GateFn.apply(s.float(), h.float(), c_scalar, c_vector)


# ------------------------------------------------------------------------------------------------
# Gaussian radial basis consumed by a linear map, formed on the fly (inference path)
# ------------------------------------------------------------------------------------------------
class _RbfLinearFn(torch.autograd.Function):
    """``h = rbf(d) W^T (+ b)`` with rbf[e,k] = exp(coeff (d_e - mu_k)^2), either formed inside the GEMM
    (``on_chip``: its splitter warps build each A tile from d and mu) or written by one elementwise
    kernel and multiplied by the plain GEMM; the basis is dropped after the product either way.  The
    backward forms d(rbf) = g W tile by tile and contracts it with d rbf / d d in the GEMM's epilogue,
    so only [E] vectors reach the distance's other consumers."""

    @staticmethod
    def fused_ok(nb, n_out):
        return PRESPLIT_WEIGHTS and 0 < nb <= 256 and nb % 4 == 0 and n_out % 4 == 0

    @staticmethod
    def forward(ctx, dist, mu, coeff, w, b, on_chip):
        lib = _lib.load()
        d = dist.contiguous()
        E, nb = d.shape[0], mu.shape[0]
        N = w.shape[0]
        ctx.save_for_backward(d, mu, w)
        ctx.coeff = float(coeff)
        ctx.fused = _RbfLinearFn.fused_ok(nb, N)
        if not ctx.fused or not on_chip:   # basis materialised for the product, then dropped
            rbf = torch.empty((E, nb), device=d.device, dtype=torch.float32)
            check(lib.e2a_rbf_fwd(ptr(d), E, ptr(mu), nb, float(coeff), ptr(rbf), stream_of(d.device)),
                  "e2a_rbf_fwd")
            return gemm(rbf, w, b)
        h = torch.empty((E, N), device=d.device, dtype=torch.float32)
        hi, lo = split_tf32(w)
        t0 = GEMM_TIMER.start()
        check(lib.e2a_gemm_tf32x3_rbf(ptr(d), ptr(mu), float(coeff), ptr(hi), ptr(lo), nb, ptr(h), N, ptr(b), E, N,
                                      nb, PASSES, stream_of(d.device)), "e2a_gemm_tf32x3_rbf")
        GEMM_TIMER.stop(t0, E, N, nb)
        return h

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            first_order_only("rbf_linear")
        lib = _lib.load()
        d, mu, w = ctx.saved_tensors
        g = g.contiguous()
        E, nb, Kh = d.shape[0], mu.shape[0], w.shape[0]
        if not ctx.fused:
            d_rbf = gemm(g, w.t().contiguous())
            dd = torch.empty_like(d)
            check(lib.e2a_rbf_bwd(ptr(d), ptr(d_rbf), E, ptr(mu), nb, ctx.coeff, ptr(dd), stream_of(d.device)),
                  "e2a_rbf_bwd")
            return dd, None, None, None, None, None
        wt = w.t().contiguous()           # [nb, Kh]: d(rbf) = g @ w
        hi, lo = split_tf32(wt)
        nblk = (nb + 63) // 64
        part = torch.empty((E, nblk), device=d.device, dtype=torch.float32)
        t0 = GEMM_TIMER.start()
        check(lib.e2a_gemm_tf32x3_rbf_dist_grad(ptr(g), Kh, ptr(hi), ptr(lo), Kh, ptr(d), ptr(mu), ctx.coeff,
                                                ptr(part), nblk, E, nb, Kh, PASSES, stream_of(d.device)),
              "e2a_gemm_tf32x3_rbf_dist_grad")
        GEMM_TIMER.stop(t0, E, nb, Kh)
        return part.sum(1), None, None, None, None, None


# Forward of the radial-basis products: False = the basis is written by one elementwise kernel and read
# by the plain GEMM (measured faster: the on-chip basis makes the GEMM's splitter warps compute one
# exponential per operand element, which they cannot do at the tensor core's rate); True = formed on
# chip.  The backward always contracts d(rbf) on chip (only [E] vectors leave the GEMM).
RBF_FWD_ON_CHIP = False


def rbf_linear(dist, mu, coeff, w, b=None, on_chip=None):
    """``GaussianSmearing(dist) @ w.T (+ b)`` (CUDA, constant weights); the basis is never kept for
    autograd."""
    return _RbfLinearFn.apply(dist.float(), mu.float().contiguous(), float(coeff), w.detach().float().contiguous(),
                              None if b is None else b.detach().float().contiguous(),
                              RBF_FWD_ON_CHIP if on_chip is None else bool(on_chip))


# ------------------------------------------------------------------------------------------------
# Per-node SO(2) map straight from positions (inference path)
# ------------------------------------------------------------------------------------------------
class NodeMapTables:
    """Host tables of the node map: J_1, J_2 (fp64), selection, CG weights, row order."""

    def __init__(self, jd, selected_idx, cg_weight, row_perm=None):
        import numpy as np

        self.j1 = np.ascontiguousarray(jd[1].detach().cpu().numpy(), dtype=np.float64)
        self.j2 = np.ascontiguousarray(jd[2].detach().cpu().numpy(), dtype=np.float64)
        self.sel = np.ascontiguousarray(np.asarray(selected_idx.detach().cpu() if hasattr(selected_idx, "cpu")
                                                   else selected_idx), dtype=np.int32)
        self.cg = np.ascontiguousarray(np.asarray(cg_weight.detach().cpu() if hasattr(cg_weight, "cpu")
                                                  else cg_weight), dtype=np.float64)
        self.perm = None if row_perm is None else np.ascontiguousarray(np.asarray(row_perm), dtype=np.int32)

    def args(self):
        import ctypes

        f = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
        return f(self.j1), f(self.j2), f(self.sel), f(self.cg), f(self.perm)


class _NodeMapFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, pos, tables):
        lib = _lib.load()
        p = pos.contiguous()
        n = p.shape[0]
        A = torch.empty((n, 20, 9), device=p.device, dtype=torch.float32)
        check(lib.e2a_node_map_fwd(ptr(p), n, *tables.args(), ptr(A), stream_of(p.device)), "e2a_node_map_fwd")
        ctx.save_for_backward(p)
        ctx.tables = tables
        return A

    @staticmethod
    def backward(ctx, g):
        if torch.is_grad_enabled():
            first_order_only("node_map_from_pos")
        lib = _lib.load()
        (p,) = ctx.saved_tensors
        g = g.contiguous()
        dp = torch.empty_like(p)
        check(lib.e2a_node_map_bwd(ptr(p), ptr(g), p.shape[0], *ctx.tables.args(), ptr(dp), stream_of(p.device)),
              "e2a_node_map_bwd")
        return dp, None


def node_map_from_pos(pos, tables):
    """[n, 20, 9] per-node SO(2) maps from positions [n, 3] (CUDA; differentiable in ``pos``)."""
    return _NodeMapFn.apply(pos.float(), tables)
