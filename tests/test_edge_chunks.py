"""Edge side in checkpointed row blocks (``edge_chunk``): the same layer output and gradients as one
block, against the reference's golden layer data, and the same energies and forces for the model."""
import json

import pytest
import torch

from golden_io import LEAVES, build_product_layer, layer_cfg, layer_inputs, load

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _run(layer, leaves, bd, Z, dout):
    out, _ = layer(node_pos=leaves["node_pos"], node_irreps_input=leaves["node_irreps_input"],
                   edge_dis=leaves["edge_dis"], edge_vec=None, attn_weight=leaves["attn_weight"], atomic_numbers=Z,
                   poly_dist=leaves["poly_dist"], batched_data=dict(bd))
    grads = torch.autograd.grad(out, [leaves[k] for k in LEAVES], dout, allow_unused=True)
    return out.detach(), grads


@pytest.mark.parametrize("name", ["layer_small_pbc", "layer_full_mol24"])
def test_layer_edge_blocks_equal_one_block(name):
    rec = load(name)
    layer = build_product_layer(layer_cfg(rec), DEV)
    leaves, bd, Z = layer_inputs(rec, DEV)
    dout = torch.tensor(rec["dout"], device=DEV)
    out1, g1 = _run(layer, leaves, bd, Z, dout)
    E = len(rec["query_idx"])
    layer.edge_chunk = max(E // 5, 1)
    assert len(layer._edge_chunks(dict(bd), len(rec["pos"]))) >= 4
    out2, g2 = _run(layer, leaves, bd, Z, dout)
    layer.edge_chunk = None
    # each row's span and radial MLP are the same arithmetic on the same operands
    assert (out1 - out2).abs().max().item() <= 1e-6 * max(out1.abs().max().item(), 1.0)
    ref = torch.tensor(rec["out"])
    assert (out2.cpu() - ref).abs().max().item() <= 1e-4 * max(ref.abs().max().item(), 1.0)
    for k, a, b in zip(LEAVES, g1, g2):
        if a is None or b is None:
            assert a is None and b is None, k
            continue
        # key-side gradients add the blocks' contributions in another order
        assert (a - b).abs().max().item() <= 1e-6 * max(a.abs().max().item(), 1.0), k
        gref = torch.tensor(rec[f"grad_{k}"])
        assert (b.cpu() - gref).abs().max().item() <= 1e-4 * max(gref.abs().max().item(), 1.0), k


def test_model_edge_blocks_equal_one_block():
    from ubio_molfm_b200.model import E2FormerPotential
    from ubio_molfm_b200.synthetic import seeded_params_

    rec = load("backbone_pbc40")
    cfg = json.loads(str(rec["cfg"]))
    seed = cfg.pop("seed")
    cfg.pop("head")
    m = E2FormerPotential(memory_saving=False, **cfg)
    seeded_params_(m.decoder, seed)
    seeded_params_(m.energy_head, seed + 1)
    m = m.to(DEV).eval()
    pos = torch.tensor(rec["pos"], device=DEV)
    Z = torch.tensor(rec["Z"], device=DEV)
    cell = torch.tensor(rec["cell"])
    pbc = [bool(v) for v in rec["pbc"]]
    e1, f1 = m(pos, Z, cell, pbc)
    g, _ = m.build_graph(pos, cell, pbc, None)
    E = g["query_idx"].numel()
    m._set_memory_mode(False, True, max(E // 4, 1))
    e2, f2 = m(pos, Z, cell, pbc)
    m._set_memory_mode(False, True, None)
    assert (e1 - e2).abs().max().item() <= 1e-6 * max(e1.abs().max().item(), 1.0)
    assert (f1 - f2).abs().max().item() <= 1e-6 * max(f1.abs().max().item(), 1.0)
    f_ref = torch.tensor(rec["forces"], dtype=torch.float64)
    assert (f2.double().cpu() - f_ref).abs().max().item() <= 1e-4
