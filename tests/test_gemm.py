"""tcgen05 3xTF32 GEMM through the C ABI against a float64 product."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (300, 200, 70), (1000, 512, 256), (4099, 1024, 1536),
                                   (7, 3, 5), (129, 130, 0), (256, 128, 1), (300, 260, 48), (200, 140, 64), (131, 129, 16)])
def test_gemm_tf32x3_matches_fp64(M, N, K):
    from ubio_molfm_b200._lib import device_status_gemm
    from ubio_molfm_b200.linear import gemm

    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn(M, K, device="cuda", generator=g)
    b = torch.randn(N, K, device="cuda", generator=g)
    bias = torch.randn(N, device="cuda", generator=g)
    ref = a.double() @ b.double().t() + bias.double()
    out = gemm(a, b, bias)
    scale = max(1.0, (K ** 0.5))
    err = (out.double() - ref).abs().max().item() / scale
    # fp32-level: within 4x the error of torch's fp32 SIMT product (plus an absolute floor)
    err32 = ((a @ b.t() + bias).double() - ref).abs().max().item() / scale
    assert err < 4 * err32 + 2e-6, (err, err32)
    out1 = gemm(a, b, bias, passes=1)
    assert (out1.double() - ref).abs().max().item() <= 2e-3 * max(1.0, ref.abs().max().item())  # plain TF32
    acc = out.clone()
    gemm(a, b, None, out=acc, accumulate=True)
    assert (acc.double() - (2 * ref - bias.double())).abs().max().item() / scale < 8 * err32 + 4e-6
    assert device_status_gemm() == 0


def test_gemm_strided_operands_and_linear_grad():
    from ubio_molfm_b200.linear import gemm, linear

    g = torch.Generator(device="cuda").manual_seed(0)
    big = torch.randn(500, 96, device="cuda", generator=g)
    a = big[:, 10:74]            # lda = 96, not 16-byte aligned start -> scalar load path
    w = torch.randn(40, 64, device="cuda", generator=g)
    ref = a.double() @ w.double().t()
    assert (gemm(a, w).double() - ref).abs().max().item() < 2e-5
    x = torch.randn(3, 70, 64, device="cuda", generator=g, requires_grad=True)
    b = torch.randn(40, device="cuda", generator=g)
    y = linear(x, w, b)
    yr = torch.nn.functional.linear(x.double(), w.double(), b.double())
    assert (y.double() - yr).abs().max().item() < 2e-5
    gy = torch.randn_like(y)
    (gx,) = torch.autograd.grad(y, x, gy)
    (gxr,) = torch.autograd.grad(yr, x, gy.double())
    assert (gx.double() - gxr).abs().max().item() < 2e-5


def test_so3_pair_product_matches_torch():
    from ubio_molfm_b200.linear import so3_pair_product

    g = torch.Generator(device="cuda").manual_seed(3)
    N, C, h = 777, 256, 192
    x = torch.randn(N, 9, C, device="cuda", generator=g, requires_grad=True)
    w1 = torch.randn(3, h, C, device="cuda", generator=g) / 16
    w2 = torch.randn(3, h, C, device="cuda", generator=g) / 16
    b = torch.randn(h, device="cuda", generator=g)
    lidx = [0, 1, 1, 1, 2, 2, 2, 2, 2]
    P = so3_pair_product(x, w1, w2, b, lidx)
    xd = x.detach().double().requires_grad_(True)
    parts = []
    for l in range(3):
        blk = xd[:, l * l:(l + 1) ** 2]
        o1 = blk @ w1[l].double().t()
        if l == 0:
            o1 = o1 + b.double()
        o2 = blk @ w2[l].double().t()
        parts.append((o1 * o2).sum(1))
    ref = torch.stack(parts, 1)
    assert (P.double() - ref).abs().max().item() <= 2e-5 * max(1.0, ref.abs().max().item())
    G = torch.randn(N, 3, h, device="cuda", generator=g)
    (dx,) = torch.autograd.grad(P, x, G)
    (dxr,) = torch.autograd.grad(ref, xd, G.double())
    assert (dx.double() - dxr).abs().max().item() <= 2e-5 * max(1.0, dxr.abs().max().item())


@pytest.mark.parametrize("M,N,K", [(300, 200, 72), (1000, 512, 256), (131, 129, 16)])
def test_gemm_general_kernel_matches_pipelined_kernel(M, N, K):
    """The register-staged kernel (unaligned rows) and the warp-specialised TMA kernel (aligned rows)
    agree with a float64 product to fp32 accuracy on the same values."""
    from ubio_molfm_b200.linear import gemm

    g = torch.Generator(device="cuda").manual_seed(7 * M + K)
    a = torch.randn(M, K, device="cuda", generator=g)
    b = torch.randn(N, K, device="cuda", generator=g)
    ref = a.double() @ b.double().t()
    out_ws = gemm(a, b)
    a_pad = torch.zeros(M, K + 1, device="cuda")
    a_pad[:, :K] = a
    out_gen = gemm(a_pad[:, :K], b)          # leading dim K + 1: not 16-byte aligned rows
    scale = max(1.0, K ** 0.5)
    err32 = ((a @ b.t()).double() - ref).abs().max().item() / scale
    for out in (out_ws, out_gen):
        assert (out.double() - ref).abs().max().item() / scale < 4 * err32 + 2e-6


def test_pair_product_recompute_matches_saved():
    """so3_pair_product with the projections formed again in the backward gives the same gradient
    as keeping them (same GEMMs, same values)."""
    from ubio_molfm_b200.linear import so3_pair_product

    g = torch.Generator(device="cuda").manual_seed(3)
    N, C, h = 300, 64, 48
    x = torch.randn(N, 9, C, device="cuda", generator=g, requires_grad=True)
    w1 = torch.randn(3, h, C, device="cuda", generator=g) / 8
    w2 = torch.randn(3, h, C, device="cuda", generator=g) / 8
    b = torch.randn(h, device="cuda", generator=g)
    lidx = [0, 1, 1, 1, 2, 2, 2, 2, 2]
    G = torch.randn(N, 3, h, device="cuda", generator=g)
    p0 = so3_pair_product(x, w1, w2, b, lidx)
    (d0,) = torch.autograd.grad(p0, x, G)
    p1 = so3_pair_product(x, w1, w2, b, lidx, recompute=True)
    (d1,) = torch.autograd.grad(p1, x, G)
    assert torch.equal(p0, p1)
    assert torch.equal(d0, d1)


def test_bounded_wait_timeout_is_reported_and_raised():
    """A bounded mbarrier wait that nothing completes (a test hook on the GEMM's own wait routine, with
    a 1 ms limit) gives up and sets the status word; the host reads it once, the potential raises after
    an evaluation that saw it, and the context stays usable."""
    from ubio_molfm_b200 import _lib
    from ubio_molfm_b200.model import E2FormerPotential
    from ubio_molfm_b200.synthetic import seeded_params_

    assert _lib.device_status_gemm(reset=True) == 0
    _lib.gemm_wait_selftest(1_000_000)
    assert _lib.device_status_gemm(reset=True) == 1
    assert _lib.device_status_gemm(reset=True) == 0
    with pytest.raises(_lib.E2AError):
        _lib.gemm_wait_selftest(10)           # limits outside [1 us, 100 ms] are refused
    m = E2FormerPotential(irreps_node_embedding="32x0e+32x1e+32x2e", num_layers=1, max_neighbors=None,
                          max_radius=4.0, number_of_basis=32, num_attn_heads=8, attn_scalar_head=8,
                          irreps_head="4x0e+4x1e+4x2e", norm_layer="rms_norm_sh", alpha_drop=0.0)
    seeded_params_(m, 1)
    m = m.cuda().eval()
    g = torch.Generator().manual_seed(0)
    pos = (torch.rand(30, 3, generator=g) * 6.0).cuda()
    Z = torch.randint(1, 9, (30,), generator=g).cuda()
    e0, f0 = m(pos, Z)
    _lib.gemm_wait_selftest(1_000_000)
    with pytest.raises(_lib.E2AError, match="timed out"):
        m(pos, Z)
    e1, f1 = m(pos, Z)                    # the word was cleared; the next evaluation is clean
    assert torch.equal(e0, e1) and torch.equal(f0, f1)


@pytest.mark.parametrize("N,C,Hd", [(1003, 256, 512), (300, 64, 64)])
def test_pair_product_backward_fused_equals_two_kernel(N, C, Hd):
    """The pair-product backward with D = pair_grad(O, G) formed inside the GEMM's A tiles
    (e2a_gemm_tf32x3_pairgrad) against the pair_grad kernel followed by the plain GEMM: the same fp32
    products are split the same way, so the input gradients are bitwise equal (ragged M included)."""
    from ubio_molfm_b200 import linear

    g = torch.Generator(device="cuda").manual_seed(N)
    x = torch.randn(N, 9, C, device="cuda", generator=g)
    w1 = torch.randn(3, Hd, C, device="cuda", generator=g) / C ** 0.5
    w2 = torch.randn(3, Hd, C, device="cuda", generator=g) / C ** 0.5
    bias = torch.randn(1, 1, Hd, device="cuda", generator=g)
    lidx = [0, 1, 1, 1, 2, 2, 2, 2, 2]
    dP = torch.randn(N, 3, Hd, device="cuda", generator=g)
    out = []
    old = linear.FUSED_PAIR_GRAD
    try:
        for fused in (True, False):
            linear.FUSED_PAIR_GRAD = fused
            xx = x.clone().requires_grad_(True)
            P = linear.so3_pair_product(xx, w1, w2, bias, lidx)
            (dx,) = torch.autograd.grad(P, xx, dP)
            out.append(dx)
    finally:
        linear.FUSED_PAIR_GRAD = old
    assert torch.equal(out[0], out[1])
