"""Row blocks of the edge side (``attention.edge_blocks``), on CPU: every edge in exactly one block, with
its own row, rows in the given spatial order, blocks near the requested edge count."""
import pytest
import torch

from ubio_molfm_b200.attention import edge_blocks


@pytest.mark.parametrize("seed,chunk,ordered", [(0, 50, True), (1, 7, False), (2, 1000, True), (3, 1, True)])
def test_edge_blocks_partition_the_edges(seed, chunk, ordered):
    g = torch.Generator().manual_seed(seed)
    n = 40
    deg = torch.randint(0, 12, (n,), generator=g)
    deg[::7] = 0                                    # rows without edges
    row_ptr = torch.nn.functional.pad(torch.cumsum(deg, 0), (1, 0)).to(torch.int32)
    E = int(row_ptr[-1])
    qi = torch.repeat_interleave(torch.arange(n), deg)
    order = torch.randperm(n, generator=g) if ordered else None
    blocks = edge_blocks(row_ptr, order, chunk)
    seen = torch.zeros(E, dtype=torch.int64)
    rows_all = []
    for rows, local, edges in blocks:
        rows_all.append(rows)
        assert bool((local[1:] >= local[:-1]).all())          # query-sorted within the block
        assert bool((qi[edges] == rows[local]).all())          # each edge sits on its own row
        for i, r in enumerate(rows.tolist()):                  # a row's edges in CSR order
            e = edges[local == i]
            assert e.tolist() == list(range(int(row_ptr[r]), int(row_ptr[r + 1])))
        seen[edges] += 1
        # a block ends at the first row that reaches its share of the edges
        assert edges.numel() <= chunk + int(deg.max()) or rows.numel() == 1
    assert bool((seen == 1).all())
    rows_all = torch.cat(rows_all)
    assert rows_all.tolist() == (order.tolist() if ordered else list(range(n)))
