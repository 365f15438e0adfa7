"""Pins the CPU oracle (oracle/) to vectors the reference itself produced.

The goldens were written by tests/golden/make_golden.py from the reference's
own sources (baseline/src/*.cpp compiled in place by oracle/Makefile). These
tests need no GPU.
"""
import hashlib
import json
import tempfile
from pathlib import Path

import numpy as np
import pytest

import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "MANIFEST.json").read_text())


def smoke1024_graph():
    import gatb200 as G
    from golden.make_golden import write_smoke1024  # the reference's prepare_smoke.py draws
    with tempfile.TemporaryDirectory() as d:
        p = Path(d) / "smoke1024.gatbin"
        write_smoke1024(p)
        assert hashlib.sha256(p.read_bytes()).hexdigest() == MANIFEST["smoke1024_gatbin_sha256"]
        return G.load_graph(p)


def test_rne_ties_and_tails():
    # baseline/tests/boundaries.cpp:25-26: midpoint ties and tails around 1.0.
    for i in range(37):
        u = np.uint32(0x3F808000 + i * 0x10000)
        x = np.array([u], np.uint32).view(np.float32)[0]
        r = O.rne(float(x))
        keep = int(u) >> 16
        rest = int(u) & 0xFFFF
        want = keep + (1 if rest > 0x8000 or (rest == 0x8000 and keep & 1) else 0)
        assert r == want
        assert O.quantize(np.array([x]))[0].view(np.uint32) == np.uint32(want << 16)


def test_degree_schedule_matches_reference():
    g = np.load(GOLDEN / "smoke1024_seed11.npz")
    graph = smoke1024_graph()
    perm, steps = O.degree_schedule(graph.row)
    assert np.array_equal(perm, g["perm"])
    assert steps == int(g["steps"][0])
    b = np.load(GOLDEN / "boundary.npz")
    perm, steps = O.degree_schedule(b["row"])
    assert np.array_equal(perm, b["perm"]) and steps == int(b["steps"][0])


def test_random_model_matches_reference(tmp_path):
    import gatb200 as G
    m = G.random_model(128, 40, 11)
    G.save_model(m, tmp_path / "w.gatwgt")
    assert hashlib.sha256((tmp_path / "w.gatwgt").read_bytes()).hexdigest() == MANIFEST["smoke1024_seed11_gatwgt_sha256"]
    om = O.random_model(128, 40, 11)
    for p, (w, al, ar, h, d) in zip(m, om):
        assert np.array_equal(p.w, w) and np.array_equal(p.al, al) and np.array_equal(p.ar, ar)


def test_config1_generator_is_deterministic(tmp_path):
    import configs
    import gatb200 as G
    cfg = configs.make("c1")
    G.save_graph(cfg.graph, tmp_path / "c1.gatbin")
    G.save_model(cfg.model, tmp_path / "c1.gatwgt")
    assert hashlib.sha256((tmp_path / "c1.gatbin").read_bytes()).hexdigest() == MANIFEST["config1_gatbin_sha256"]
    assert hashlib.sha256((tmp_path / "c1.gatwgt").read_bytes()).hexdigest() == MANIFEST["config1_gatwgt_sha256"]
    deg = np.diff(cfg.graph.row.astype(np.int64))
    assert cfg.graph.e == 16384 and np.all(deg == 16)


@pytest.mark.parametrize("name", ["smoke1024_seed11", "config1"])
def test_ref_chain_matches_reference(name):
    """R0 restatement vs the reference's R0 (FP32; only summation order differs)."""
    import configs
    import gatb200 as G
    g = np.load(GOLDEN / f"{name}.npz")
    if name == "config1":
        cfg = configs.make("c1")
        graph, model = cfg.graph, [(p.w, p.al, p.ar, p.heads, p.dim) for p in cfg.model]
    else:
        graph, model = smoke1024_graph(), O.random_model(128, 40, 11)
    outs = O.ref_chain(graph.row, graph.col, graph.x, model)
    for l, o in enumerate(outs, 1):
        for s in ("left", "right", "max", "den"):
            ref = g[f"ref_l{l}_{s}"]
            tol = 1e-5 * max(1.0, float(np.abs(ref).max()))
            assert np.abs(o[s] - ref).max() <= tol, (l, s)
    e = O.errors(g["ref_logits"], outs[2]["out"])
    assert e["max_abs"] <= 1e-5, e


def test_fp64_oracle_vs_reference_r0():
    """boundaries.cpp:30 gate: R0 within 1e-4 of the FP64 oracle."""
    b = np.load(GOLDEN / "boundary.npz")
    for D in (17, 128):
        row, col, x = O.boundary_graph(D)
        for K in (1, 8):
            for d in (7, 47):
                w, al, ar = O.boundary_params(D, K, d)
                out = O.fp64_layer(row, col, x, w, al, ar, K, d)
                e = O.errors(out, b[f"ref_{D}_{K}_{d}"])
                assert e["max_abs"] < 1e-4 and e["relative_l2"] < 1e-4


@pytest.mark.parametrize("D", [17, 33, 128, 256])
def test_boundary_cases_match_reference(D):
    b = np.load(GOLDEN / "boundary.npz")
    row, col, x = O.boundary_graph(D)
    assert np.array_equal(row, b["row"]) and np.array_equal(col, b["col"])
    for K in (1, 2, 4, 8):
        for d in (7, 32, 40, 47):
            key = f"{D}_{K}_{d}"
            w, al, ar = O.boundary_params(D, K, d)
            sums = b["wsum_" + key]
            assert np.array_equal([w.astype(np.float64).sum(), al.astype(np.float64).sum(),
                                   ar.astype(np.float64).sum()], sums)
            o = O.ref_layer(row, col, x, w, al, ar, K, d, False)
            e = O.errors(b["ref_" + key], o["out"])
            assert e["max_abs"] <= 1e-5, (key, e)
            # empty rows produce exact zeros (boundaries.cpp:33)
            assert np.all(o["out"][0] == 0)
            if "b0bf16_" + key in b:
                bo = O.b0_layer(row, col, x, w, al, ar, K, d, False, bf16=True)
                e = O.errors(b["b0bf16_" + key], bo["out"])
                assert e["max_abs"] <= 2e-5, (key, e)


def test_b0_chain_matches_reference():
    g = np.load(GOLDEN / "config1.npz")
    import configs
    cfg = configs.make("c1")
    inp = cfg.graph.x
    for l, p in enumerate(cfg.model):
        o = O.b0_layer(cfg.graph.row, cfg.graph.col, inp, p.w, p.al, p.ar, p.heads, p.dim, l < 2, bf16=True)
        inp = o["out"]
    e = O.errors(g["b0bf16_logits"], inp)
    # Each layer re-rounds its input to BF16 (convert, common.cpp:85-93): an FP32
    # difference in the last bits can flip one BF16 rounding (2^-9 relative),
    # so the chained B0 restatement agrees to ~4e-5, not to FP32 precision.
    # For scale: B0 BF16 itself is 2.8e-3 (rel-L2) away from R0 on this input.
    assert e["relative_l2"] <= 2e-4, e
