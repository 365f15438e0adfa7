"""Seeded synthetic stand-ins for the benchmark configurations.

The reference measures on ogbn-arxiv / ogbn-products GATBIN1 files that are not
available here. These configurations reproduce their shapes (node and edge
counts, degree tails, feature widths, classes) with seeded generators
(gat_b200_synth_*), so every run builds bit-identical inputs.

  c1  tiny: 1,024 nodes, 15 uniform distinct sources + self loop per row,
      X ~ N(0,1) 1024x128, 128 -> 8x32 -> 8x32 -> 1x40, Glorot weights.
  c2  arxiv-like: 169,343 nodes, 2,484,941 edges incl. self loops, power-law
      degrees (gamma 2.1, max 13,162), X ~ N(0,1) x128, classes 40.
  c3  layer-2 micro on the c2 graph: H ~ N(0,1) 169,343x256, a ~ U(-0.1,0.1),
      W 256x256 Glorot.
  c4  products-like: 2,449,029 nodes, 126,167,053 edges incl. self loops,
      power-law degrees (gamma 2.1, max 17,482), X ~ N(0,1) x100, classes 47.
  c4s c4 scaled down 4x (profiler captures only).
  c5  RMAT stress: RMAT(a=.57, b=.19, c=.19, d=.05) over 2^24 nodes with
      2^29 edge draws, self loops, duplicates merged (destination-row CSR),
      X ~ N(0,1) x256, 256 -> 8x32 -> 8x32 -> 1x64. Generated on the GPU
      (gat_b200_synth_rmat).
  c5s c5 scaled down 16x (2^20 nodes, 2^25 draws) for tests and profiles.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import gatb200 as G

SPECS = {
    "c1": dict(kind="uniform", n=1024, sources=15, din=128, classes=40, seed=1),
    "c2": dict(kind="powerlaw", n=169_343, e=2_484_941, max_degree=13_162, gamma=2.1, din=128, classes=40, seed=2),
    "c4": dict(kind="powerlaw", n=2_449_029, e=126_167_053, max_degree=17_482, gamma=2.1, din=100, classes=47, seed=4),
    # c4 scaled down 4x in nodes and edges (same mean degree and model) for
    # profiler captures: its features (0.3 GB per layer) still exceed L2.
    "c4s": dict(kind="powerlaw", n=612_257, e=31_541_763, max_degree=8_000, gamma=2.1, din=100, classes=47, seed=4),
    "c5": dict(kind="rmat", log2n=24, draws=1 << 29, a=0.57, b=0.19, c=0.19, din=256, classes=64, seed=5),
    "c5s": dict(kind="rmat", log2n=20, draws=1 << 25, a=0.57, b=0.19, c=0.19, din=256, classes=64, seed=5),
}


def _rmat(s, r_lo=0, r_hi=None, cols=True):
    return G.synth_rmat(s["log2n"], s["draws"], s["a"], s["b"], s["c"], s["seed"], r_lo, r_hi, cols)


@dataclass
class Config:
    name: str
    graph: G.Graph
    model: list


def make_graph(name: str, features: bool = True) -> G.Graph:
    s = SPECS[name]
    if s["kind"] == "uniform":
        row, col = G.synth_uniform_graph(s["n"], s["sources"], s["seed"])
    elif s["kind"] == "rmat":
        row, col = _rmat(s)
    else:
        row, col = G.synth_powerlaw_graph(s["n"], s["e"], s["max_degree"], s["gamma"], s["seed"])
    n = len(row) - 1
    x = G.synth_normal((n, s["din"]), s["seed"], 1) if features else np.zeros((0, s["din"]), np.float32)
    return G.Graph(n, len(col), s["din"], s["classes"], row, col, x)


def make(name: str, features: bool = True) -> Config:
    s = SPECS[name]
    return Config(name, make_graph(name, features), G.glorot_model(s["din"], s["classes"], s["seed"]))


@dataclass
class Part:
    """This rank's share of a power-law configuration (multi-GPU runs)."""
    name: str
    row: np.ndarray      # all n+1 row pointers
    col_rows: np.ndarray  # sources of rows [lo, hi)
    x_rows: np.ndarray    # features of rows [lo, hi)
    cuts: np.ndarray
    lo: int
    hi: int
    e: int
    din: int
    model: list


def make_part(name: str, rank: int, world: int) -> Part:
    """Generates only what rank `rank` of `world` needs: every rank builds the
    row pointers, then the sources and features of its own rows (the rows of
    gat_b200_partition's cut, as the partitioned model takes them)."""
    s = SPECS[name]
    if s["kind"] == "powerlaw":
        row = G.synth_powerlaw_rowptr(s["n"], s["e"], s["max_degree"], s["gamma"], s["seed"])
    elif s["kind"] == "rmat":
        row, _ = _rmat(s, cols=False)  # generated on this rank's GPU
    else:
        raise ValueError("make_part needs a power-law or RMAT configuration")
    cuts = G.partition(row, world)[0]
    lo, hi = int(cuts[rank]), int(cuts[rank + 1])
    if s["kind"] == "rmat":
        _, col = _rmat(s, lo, hi)
    else:
        col = G.synth_powerlaw_cols(s["n"], s["e"], s["max_degree"], s["gamma"], s["seed"], row, lo, hi)
    x = G.synth_normal_range(lo * s["din"], (hi - lo, s["din"]), s["seed"], 1)
    return Part(name, row, col, x, cuts, lo, hi, int(row[-1]), s["din"],
                G.glorot_model(s["din"], s["classes"], s["seed"]))
