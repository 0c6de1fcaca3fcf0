"""Double backward (``create_graph=True``) for force-loss training.

The reference gives each kernel-level sparse op a differentiable backward (``*Backward_Fn``:
triton_sparse_qk_autograd.py:754-836, sparse_alpha_sum_edge_index_autograd.py:173-208,
sparse_v_agg_edge_index_cblocked_bench.py:361-420, edge_degree_outer_autograd.py:259-296), so that a
loss on forces = -dE/dpos can be back-propagated to the parameters.  Checked here:

* each kernel-level op: first- and second-order gradients (w.r.t. every input and the upstream
  gradient) against the same procedure on the oracle's float64 PyTorch restatement;
* the fused attention span (its create_graph backward goes through the kernel-level ops);
* the whole model in training mode: parameter gradients of ``E^2 + sum F^2`` against the float64
  oracle model on the same weights and graph.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _second_order(fn, inputs, seed):
    """First-order grads of <fn(x), w> and the grads of <first-order grads, r> w.r.t. (x, w)."""
    g = torch.Generator().manual_seed(seed)
    y = fn(*inputs)
    w = torch.randn(y.shape, generator=g, dtype=torch.float64).to(y.device, y.dtype).requires_grad_(True)
    first = torch.autograd.grad(y, inputs, w, create_graph=True)
    rs = [torch.randn(f.shape, generator=g, dtype=torch.float64).to(f.device, f.dtype) for f in first]
    z = sum((f * r).sum() for f, r in zip(first, rs))
    second = torch.autograd.grad(z, list(inputs) + [w], allow_unused=True)
    return [t.detach() for t in first], [None if t is None else t.detach() for t in second]


def _leaves(tensors):
    cpu = [t.double().requires_grad_(True) for t in tensors]
    dev = [t.float().to(DEV).requires_grad_(True) for t in tensors]
    return cpu, dev


def _close(a, b, rel, what):
    if a is None or b is None:
        za = a is None or float(a.abs().max()) == 0.0
        zb = b is None or float(b.abs().max()) == 0.0
        assert za and zb, what
        return
    a = a.double().cpu()
    scale = max(float(b.abs().max()), 1e-12)
    err = float((a - b).abs().max())
    assert err <= rel * scale, f"{what}: max err {err:.3e} vs scale {scale:.3e}"


def _graph(seed, N=60, M=80, E=700):
    g = torch.Generator().manual_seed(seed)
    qi = torch.sort(torch.randint(0, N, (E,), generator=g)).values
    ki = torch.randint(0, M, (E,), generator=g)
    return g, qi, ki, N, M, E


def test_sparse_qk_double_backward_matches_oracle():
    from oracle import attention_ref as R
    from ubio_molfm_b200.ops import prepare_sparse_qk_edge_index_metadata, sparse_qk_edge_index_triton

    g, qi, ki, N, M, E = _graph(1)
    H, D = 8, 16
    q0, k0 = torch.randn(N, H, D, generator=g), torch.randn(M, H, D, generator=g)
    md = prepare_sparse_qk_edge_index_metadata(qi.to(DEV), ki.to(DEV), N, M)
    (qc, kc), (qd, kd) = _leaves([q0, k0])
    f_ref, s_ref = _second_order(lambda q, k: R.sparse_qk(q, k, qi, ki), [qc, kc], 5)
    f_dev, s_dev = _second_order(lambda q, k: sparse_qk_edge_index_triton(q, k, qi.to(DEV), ki.to(DEV), md),
                                 [qd, kd], 5)
    for i, (a, b) in enumerate(zip(f_dev, f_ref)):
        _close(a, b, 1e-5, f"first-order {i}")
    for i, (a, b) in enumerate(zip(s_dev, s_ref)):
        _close(a, b, 1e-5, f"second-order {i}")


def test_v_agg_double_backward_matches_oracle():
    from oracle import attention_ref as R
    from ubio_molfm_b200.ops import prepare_sparse_qk_edge_index_metadata, sparse_v_agg_edge_index_triton_cblocked

    g, qi, ki, N, M, E = _graph(2)
    C, H = 12, 8
    v0, a0 = torch.randn(M, C, H, generator=g), torch.randn(E, H, generator=g)
    md = prepare_sparse_qk_edge_index_metadata(qi.to(DEV), ki.to(DEV), N, M)
    (vc, ac), (vd, ad) = _leaves([v0, a0])
    f_ref, s_ref = _second_order(lambda v, a: R.v_agg(v, a, qi, ki, N), [vc, ac], 6)
    f_dev, s_dev = _second_order(
        lambda v, a: sparse_v_agg_edge_index_triton_cblocked(v, a, qi.to(DEV), ki.to(DEV), N, md), [vd, ad], 6)
    for i, (a, b) in enumerate(zip(f_dev, f_ref)):
        _close(a, b, 1e-5, f"first-order {i}")
    for i, (a, b) in enumerate(zip(s_dev, s_ref)):
        _close(a, b, 1e-5, f"second-order {i}")


def test_alpha_sum_double_backward_matches_oracle():
    from oracle import attention_ref as R
    from ubio_molfm_b200.ops import sparse_alpha_sum_edge_index_triton

    g, qi, _, N, _, E = _graph(3)
    H = 8
    (ac,), (ad,) = _leaves([torch.randn(E, H, generator=g)])
    # the sum is linear: its second-order terms w.r.t. alpha vanish and only d/d(upstream) remains
    f_ref, s_ref = _second_order(lambda a: R.alpha_sum(a, qi, N) ** 2, [ac], 7)
    f_dev, s_dev = _second_order(lambda a: sparse_alpha_sum_edge_index_triton(a, qi.to(DEV), N) ** 2, [ad], 7)
    for i, (a, b) in enumerate(zip(f_dev, f_ref)):
        _close(a, b, 1e-5, f"first-order {i}")
    for i, (a, b) in enumerate(zip(s_dev, s_ref)):
        _close(a, b, 1e-5, f"second-order {i}")


@pytest.mark.parametrize("L,F", [(9, 128), (5, 24)])
def test_edge_degree_outer_double_backward_matches_oracle(L, F):
    from oracle import attention_ref as R
    from ubio_molfm_b200.ops import edge_degree_outer_triton

    g, qi, _, N, _, E = _graph(4)
    (shc, fec), (shd, fed) = _leaves([torch.randn(E, L, generator=g), torch.randn(E, F, generator=g)])
    f_ref, s_ref = _second_order(lambda s, f: R.edge_outer(s, f, qi, N), [shc, fec], 8)
    f_dev, s_dev = _second_order(lambda s, f: edge_degree_outer_triton(s, f, qi.to(DEV), N), [shd, fed], 8)
    for i, (a, b) in enumerate(zip(f_dev, f_ref)):
        _close(a, b, 1e-5, f"first-order {i}")
    for i, (a, b) in enumerate(zip(s_dev, s_ref)):
        _close(a, b, 1e-5, f"second-order {i}")


@pytest.mark.parametrize("H,D,C", [(8, 4, 20), (128, 8, 58)])
def test_attention_span_double_backward_matches_oracle(H, D, C):
    from oracle import attention_ref as R
    from ubio_molfm_b200.ops import attention_span, prepare_sparse_qk_edge_index_metadata

    g, qi, ki, N, M, E = _graph(9, N=50, M=70, E=600)
    md = prepare_sparse_qk_edge_index_metadata(qi.to(DEV), ki.to(DEV), N, M)
    vals = [torch.randn(N, H, D, generator=g) * 0.5, torch.randn(M, H, D, generator=g) * 0.5,
            torch.randn(M, C, H, generator=g), torch.randn(E, 2 * H, generator=g),
            torch.rand(E, generator=g) * 0.9 + 0.1, torch.rand(E, generator=g) * 4 + 0.8]
    cpu, dev = _leaves(vals)
    f_ref, s_ref = _second_order(lambda *x: R.attention_span(*x, qi, ki, N), cpu, 10)
    f_dev, s_dev = _second_order(lambda *x: attention_span(*x, md, keep_logits=True), dev, 10)
    names = ["q", "k", "v", "gate", "poly", "dist", "upstream"]
    for n, a, b in zip(names, f_dev, f_ref):
        _close(a, b, 2e-5, f"first-order d{n}")
    for n, a, b in zip(names, s_dev, s_ref):
        _close(a, b, 1e-4, f"second-order d{n}")


def test_attention_span_double_backward_with_dependent_inputs():
    """As in the model, the envelope and the radial gate are functions of the distance: the span's
    create_graph backward must return partial derivatives, not the total derivative through dist."""
    from oracle import attention_ref as R
    from ubio_molfm_b200.ops import attention_span, prepare_sparse_qk_edge_index_metadata

    H, D, C = 8, 8, 116
    g, qi, ki, N, M, E = _graph(11, N=50, M=70, E=600)
    md = prepare_sparse_qk_edge_index_metadata(qi.to(DEV), ki.to(DEV), N, M)
    vals = [torch.randn(N, H, D, generator=g) * 0.5, torch.randn(M, H, D, generator=g) * 0.5,
            torch.randn(M, C, H, generator=g), torch.randn(E, 2 * H, generator=g),
            torch.rand(E, generator=g) * 4 + 0.8]
    cpu, dev = _leaves(vals)

    def composed(span):
        def fn(q, k, v, g0, d):
            poly = 0.5 * (torch.cos(d * 0.5) + 1.0)
            gate = g0 * torch.tanh(d).unsqueeze(-1)
            return span(q, k, v, gate, poly, d)
        return fn

    f_ref, s_ref = _second_order(composed(lambda *x: R.attention_span(*x, qi, ki, N)), cpu, 12)
    f_dev, s_dev = _second_order(composed(lambda *x: attention_span(*x, md)), dev, 12)
    names = ["q", "k", "v", "gate0", "dist", "upstream"]
    for n, a, b in zip(names, f_dev, f_ref):
        _close(a, b, 2e-5, f"first-order d{n}")
    for n, a, b in zip(names, s_dev, s_ref):
        _close(a, b, 1e-4, f"second-order d{n}")


def test_eval_mode_fused_path_refuses_create_graph():
    """The inference-only fused ops raise instead of returning gradients without their second-order part."""
    from ubio_molfm_b200.linear import rms_norm

    x = torch.randn(10, 9, 128, device=DEV, requires_grad=True)
    y = rms_norm(x, torch.ones(3, 128, device=DEV), torch.zeros(128, device=DEV), 1e-5)
    with pytest.raises(RuntimeError, match="double backward"):
        torch.autograd.grad(y.square().sum(), x, create_graph=True)


SMALL = dict(irreps_node_embedding="32x0e+32x1e+32x2e", num_layers=2, max_neighbors=None, max_radius=5.0,
             number_of_basis=32, num_attn_heads=8, attn_scalar_head=8, irreps_head="4x0e+4x1e+4x2e",
             norm_layer="rms_norm_sh", alpha_drop=0.0, tp_type="QK_alpha", attn_type="so2-first-order",
             atom_type_cnt=256, avg_degree=23.0)


def test_force_loss_parameter_gradients_match_oracle():
    """Training mode: forces keep their graph (create_graph = training, as the reference's force head),
    and the parameter gradients of E^2 + sum |F|^2 match the float64 oracle model's on the same graph."""
    from oracle import graph_ref
    from oracle import model_ref as M
    from ubio_molfm_b200.graph import pbc_image_offsets
    from ubio_molfm_b200.model import E2FormerPotential
    from ubio_molfm_b200.synthetic import seeded_params_

    rng = np.random.default_rng(12)
    L = 7.0
    n = 40
    pos = (rng.random((n, 3)) * L).astype(np.float32)
    Z = torch.tensor(rng.choice([1, 6, 7, 8], n))
    cell = np.eye(3, dtype=np.float32) * L

    model = E2FormerPotential(**SMALL)
    seeded_params_(model.decoder, 31)
    seeded_params_(model.energy_head, 32)
    p = {k: v.detach().clone().double().requires_grad_(v.is_floating_point())
         for k, v in model.decoder.state_dict().items()}
    ph = {k: v.detach().clone().double().requires_grad_(True) for k, v in model.energy_head.state_dict().items()}
    model = model.to(DEV).train()

    # CUDA model, training mode
    energy, forces = model(torch.tensor(pos, device=DEV), Z.to(DEV), torch.tensor(cell), (True, True, True))
    assert forces.requires_grad and energy.requires_grad
    loss = energy.square().sum() + forces.square().sum()
    named = [("d", k, t) for k, t in model.decoder.named_parameters() if t.requires_grad] + \
            [("h", k, t) for k, t in model.energy_head.named_parameters()]
    grads = torch.autograd.grad(loss, [t for _, _, t in named], allow_unused=True)

    # float64 oracle on the same graph
    off = pbc_image_offsets(cell, [True, True, True], SMALL["max_radius"]).numpy()
    ia = graph_ref.pbc_expand(pos, off, SMALL["max_radius"])
    outcell, offsets = ia % n, off[ia // n]
    exp = (pos[outcell] + offsets).astype(np.float32)
    qi, ni, _ = graph_ref.radius_graph(pos, exp, [0, n], [0, len(exp)], SMALL["max_radius"], 1e-4, None)
    qi, ni, outcell = torch.tensor(qi), torch.tensor(ni), torch.tensor(outcell)
    pd = torch.tensor(pos, dtype=torch.float64, requires_grad=True)
    exp_pos = pd[outcell] + torch.tensor(offsets, dtype=torch.float64)
    cfg = dict(SMALL)
    x = M.backbone(p, cfg, pd, Z, qi, ni, outcell, exp_pos, True)
    h = torch.nn.functional.silu(torch.nn.functional.linear(x[:, 0], ph["mlp.0.weight"], ph["mlp.0.bias"]))
    h = torch.nn.functional.silu(torch.nn.functional.linear(h, ph["mlp.2.weight"], ph["mlp.2.bias"]))
    e_ref = torch.nn.functional.linear(h, ph["mlp.4.weight"], ph["mlp.4.bias"]).sum()
    (gpos,) = torch.autograd.grad(e_ref, pd, create_graph=True)
    loss_ref = e_ref.square() + gpos.square().sum()
    # training-mode forces (computed with a graph) equal the oracle's first-order forces
    assert float((forces.detach().double().cpu() + gpos.detach()).abs().max()) <= 1e-6
    assert abs(float(loss.detach()) - float(loss_ref.detach())) <= 1e-5 * abs(float(loss_ref.detach()))
    ref_leaves = [(p if src == "d" else ph)[k] for src, k, _ in named]
    ref_grads = torch.autograd.grad(loss_ref, ref_leaves, allow_unused=True)
    num = den = 0.0
    for (_, k, _), a, b in zip(named, grads, ref_grads):
        if b is None:
            assert a is None or float(a.abs().max()) == 0.0, k
            continue
        assert a is not None, f"{k}: no gradient on the CUDA path"
        d = a.double().cpu() - b
        num += float(d.square().sum())
        den += float(b.square().sum())
        _close(a, b, 1e-4, k)
    assert (num / den) ** 0.5 <= 5e-5, (num / den) ** 0.5
