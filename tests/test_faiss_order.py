"""The expanded-node order of the reference's FAISS neighbour path (``use_faiss=True``).

``distributed_cell_expand`` is pinned bit-exactly to the reference's own function (fixtures
``faiss_expand_*.npz`` made by running it on CPU), and a radius graph over that expansion holds the
same physical edges, with the same distances, as one over ``CellExpander``'s expansion (both built
by the C graph oracle).  FAISS itself (its top-k tie order) is not part of this: parity unpinned."""
import numpy as np
import pytest
import torch

from golden_io import load

CASES = ["faiss_expand_water648", "faiss_expand_triclinic60", "faiss_expand_small40"]


def _expand(rec):
    from ubio_molfm_b200.graph import distributed_cell_expand

    pos = torch.tensor(rec["pos"]).unsqueeze(0)
    return distributed_cell_expand(pos, torch.tensor(rec["cell"]), float(rec["cutoff"]), pos[0].min(dim=0)[0],
                                   pos[0].max(dim=0)[0], 1, torch.tensor(rec["pbc"]).reshape(1, 3))


@pytest.mark.parametrize("name", CASES)
def test_distributed_cell_expand_bit_exact(name):
    rec = load(name)
    out = _expand(rec)
    assert out["expand_node_pos"].shape[0] == 1 and bool(out["expand_node_mask"].all())
    np.testing.assert_array_equal(out["outcell_index"][0].numpy(), rec["outcell_index"])
    np.testing.assert_array_equal(out["expand_node_pos"][0].numpy(), rec["expand_node_pos"])


def test_distributed_cell_expand_argument_errors():
    from ubio_molfm_b200.graph import distributed_cell_expand

    with pytest.raises(ValueError):
        distributed_cell_expand(torch.zeros(5, 3), torch.eye(3), 1.0, torch.zeros(3), torch.ones(3))
    with pytest.raises(ValueError):
        distributed_cell_expand(torch.zeros(2, 5, 3), torch.eye(3), 1.0, torch.zeros(3), torch.ones(3))
    out = distributed_cell_expand(torch.zeros(1, 5, 3), torch.eye(3), 1.0, torch.zeros(3), torch.ones(3), pbc=None)
    assert out["expand_node_pos"].shape == (1, 5, 3)


@pytest.mark.parametrize("name", ["faiss_expand_water648", "faiss_expand_small40"])
def test_faiss_order_graph_has_the_same_edges(name):
    from oracle import graph_ref
    from ubio_molfm_b200.graph import pbc_image_offsets

    rec = load(name)
    pos, cutoff = rec["pos"].astype(np.float32), float(rec["cutoff"])
    n = len(pos)
    out = _expand(rec)
    exp_f = out["expand_node_pos"][0].numpy()
    oc_f = out["outcell_index"][0].numpy()
    off = pbc_image_offsets(rec["cell"], [bool(v) for v in rec["pbc"]], cutoff).numpy()
    ia = graph_ref.pbc_expand(pos, off, cutoff)
    oc_c = ia % n
    exp_c = (pos[oc_c] + off[ia // n]).astype(np.float32)

    def edges(exp, oc):
        qi, ni, dist = graph_ref.radius_graph(pos, exp, [0, n], [0, len(exp)], cutoff, 1e-4, None)
        # a physical edge: (query atom, neighbour atom, image position rounded to 1e-4 A), with its distance
        key = np.round(exp[ni] * 1e4).astype(np.int64)
        return sorted(zip(qi.tolist(), oc[ni].tolist(), map(tuple, key.tolist()), dist.tolist()))

    ef, ec = edges(exp_f, oc_f), edges(exp_c, oc_c)
    assert len(ef) == len(ec) > 0
    assert ef == ec
