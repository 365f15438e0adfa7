"""RMAT stress configuration (c5): generator and sampled FP64 parity.

* gat_b200_synth_rmat (GPU) equals a numpy restatement of the same
  counter-based draws, quadrant rule, self loops and de-duplication, bit for
  bit, on small graphs.
* A full R0 oracle of c5 (2^24 nodes, ~0.5 G edges) does not fit the host, so
  each layer is checked on sampled rows with their complete neighbourhoods
  (tests/sampled_fp64.py). Gate: relative L2 over all sampled rows <= 1e-2
  (the BF16 gate against R0), <= 3e-2 for every row.
"""
import numpy as np
import pytest

import configs
import gatb200 as G
from sampled_fp64 import sampled_forward_check

pytestmark = pytest.mark.gpu

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def _splitmix(x):
    x = x + np.uint64(0x9E3779B97F4A7C15)
    x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return x ^ (x >> np.uint64(31))


def _rmat_numpy(lg, draws, a, b, c, seed):
    """Restatement of the generator: level l of edge k draws
    unit(splitmix64(base + k*lg + l)), base = splitmix64(seed ^ splitmix64(7 + C))."""
    with np.errstate(over="ignore"):
        base = _splitmix(np.uint64(seed) ^ _splitmix(np.uint64(7) + np.uint64(0x632BE59BD9B4E019)))
        k = np.arange(draws, dtype=np.uint64)
        src = np.zeros(draws, np.uint64)
        dst = np.zeros(draws, np.uint64)
        for lev in range(lg):
            u = (_splitmix(base + k * np.uint64(lg) + np.uint64(lev)) >> np.uint64(11)).astype(np.float64) \
                * (1.0 / 9007199254740992.0)
            bs = (u >= a + b).astype(np.uint64)
            bd = (((u >= a) & (u < a + b)) | (u >= a + b + c)).astype(np.uint64)
            src = (src << np.uint64(1)) | bs
            dst = (dst << np.uint64(1)) | bd
    n = 1 << lg
    ids = np.arange(n, dtype=np.uint64)
    keys = np.unique(np.concatenate([(dst << np.uint64(lg)) | src, (ids << np.uint64(lg)) | ids]))
    row = np.searchsorted(keys, ids << np.uint64(lg), side="left").astype(np.uint64)
    row = np.append(row, np.uint64(len(keys)))
    col = (keys & np.uint64(n - 1)).astype(np.uint32)
    return row, col


@pytest.mark.parametrize("lg,draws,seed", [(6, 500, 1), (10, 20_000, 5), (14, 300_000, 9)])
def test_rmat_generator_matches_restatement(dev, lg, draws, seed):
    row, col = G.synth_rmat(lg, draws, 0.57, 0.19, 0.19, seed)
    want_row, want_col = _rmat_numpy(lg, draws, 0.57, 0.19, 0.19, seed)
    assert np.array_equal(row, want_row)
    assert np.array_equal(col, want_col)
    G.Graph(len(row) - 1, len(col), 1, 1, row, col, np.zeros((len(row) - 1, 1), np.float32)).validate()
    # a row range returns the same sources
    lo, hi = (1 << lg) // 3, (1 << lg) // 2
    _, part = G.synth_rmat(lg, draws, 0.57, 0.19, 0.19, seed, lo, hi)
    assert np.array_equal(part, col[int(row[lo]):int(row[hi])])


def test_rmat_generator_argument_checks(dev):
    with pytest.raises(G.GatError, match="a\\+b\\+c"):
        G.synth_rmat(10, 100, 0.5, 0.3, 0.3, 1)
    with pytest.raises(G.GatError, match="2\\^31"):
        G.synth_rmat(30, 1 << 31, 0.57, 0.19, 0.19, 1, cols=False)


@pytest.mark.parametrize("name", ["c5s", "c5"])
def test_rmat_sampled_rows_fp64(dev, name):
    r = sampled_forward_check(configs.make(name))
    assert r["rel_l2"] <= 1e-2, (name, r)
    assert r["worst"][3] <= 3e-2, (name, r)
