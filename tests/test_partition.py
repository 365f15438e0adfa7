"""The C++ row partition of the multi-GPU forward (gat_b200_partition,
gat_b200_partition_slots, used by gat_b200_part_model_create) against the
Python layout the CPU gloo tests run the oracle through (dist.Layout): the
same rank cuts, chunk cuts, block size and table rows, bit for bit, on
graphs with empty rows, hubs larger than a rank's share, and more ranks or
chunks than rows."""
import numpy as np
import pytest

import configs
import dist as gdist
import gatb200 as G


def _graphs():
    yield "c1", configs.make_graph("c1", features=False).row, configs.make_graph("c1", features=False).col
    row, col = G.synth_powerlaw_graph(20000, 400000, 9000, 2.1, 5)
    yield "powerlaw", row, col
    # a hub that holds most edges, empty rows around it
    deg = np.zeros(50, np.int64)
    deg[7] = 900
    deg[[0, 3, 40]] = [5, 2, 1]
    row = np.concatenate([[0], np.cumsum(deg)]).astype(np.uint64)
    rng = np.random.default_rng(3)
    col = np.concatenate([np.sort(rng.choice(50, size=min(d, 50), replace=False)) if d <= 50 else
                          np.sort(rng.integers(0, 50, size=d)) for d in deg]).astype(np.uint32)
    yield "hub", row, col
    yield "tiny", np.array([0, 1, 1, 3], np.uint64), np.array([0, 1, 2], np.uint32)


@pytest.mark.parametrize("world,chunks", [(1, 1), (2, 1), (2, 4), (4, 3), (8, 1), (8, 2), (3, 7)])
def test_partition_matches_python_layout(world, chunks):
    for name, row, col in _graphs():
        cuts, cc, block_rows, table_rows = G.partition(row, world, chunks)
        lay = gdist.Layout(row, world, chunks)
        assert np.array_equal(cuts, lay.cuts), (name, cuts, lay.cuts)
        assert np.array_equal(cc, lay.ccuts), name
        assert block_rows == lay.chunk_max and table_rows == lay.n_table, name
        got = G.partition_slots(row, world, chunks, col)
        assert np.array_equal(got, lay.slots(col)), name
        # every table row is hit by at most one source id, and it lies in the block of its owner
        n = len(row) - 1
        ids = np.arange(n, dtype=np.uint32)
        s = G.partition_slots(row, world, chunks, ids)
        assert len(np.unique(s)) == n and int(s.max()) < table_rows


def test_partition_rejects_bad_input():
    row = np.array([0, 2, 1], np.uint64)
    with pytest.raises(G.GatError, match="nonmonotone CSR"):
        G.partition(row, 2)
    with pytest.raises(G.GatError, match="world size"):
        G.partition(np.array([0, 1], np.uint64), 9)
    with pytest.raises(G.GatError, match="source index out of bounds"):
        G.partition_slots(np.array([0, 1, 2], np.uint64), 2, 1, np.array([5], np.uint32))
