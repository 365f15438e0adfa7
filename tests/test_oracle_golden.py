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


TFS_CASES = [(17, 1, 7), (33, 2, 40), (128, 8, 32), (256, 8, 32), (256, 1, 47), (128, 4, 47)]


@pytest.mark.parametrize("case", TFS_CASES, ids=lambda c: "_".join(map(str, c)))
def test_tfs_family_matches_reference(case):
    """TFS restatements vs the reference's own B1 / icpp_online / icpp_block /
    icpp_heads_hybrid on the same inputs (L, R, max from the reference).

    The reference accumulates V = sum RNE(.) x W with AMX tdpbf16ps, whose
    internal summation does not reproduce as sequential FP32 adds: the
    restatement agrees to ~1e-5 relative, not bit for bit. den (plain FP32
    sums of the same exp values) is exact."""
    D, K, d = case
    key = f"{D}_{K}_{d}"
    t = np.load(GOLDEN / "tfs.npz")
    row, col, x = O.boundary_graph(D)
    w, al, ar = O.boundary_params(D, K, d)
    xq, wq = O.quantize(x), O.quantize(w)
    L, R, mx = t["lbf_" + key], t["rbf_" + key], t["max_" + key]

    def close(got, want, rel):
        scale = max(1e-30, float(np.abs(want).max()))
        assert np.abs(got - want).max() <= rel * scale, (key, float(np.abs(got - want).max() / scale))

    blr = O.prepare_blr(w, al, ar, K, d)
    close(blr, t["blr_" + key], 1e-6)
    l0, r0 = O.lr_reordered(x, t["blr_" + key], K, 0)
    close(np.concatenate([l0, r0]), np.concatenate([L, R]), 1e-4)  # oneMKL BF16 GEMM order
    l1, r1 = O.lr_reordered(x, t["blr_" + key], K, 1)
    close(np.concatenate([l1, r1]), np.concatenate([t["l32_" + key], t["r32_" + key]]), 2e-6)
    assert np.array_equal(O.max_prescan(row, col, L, R, K), mx)

    out, den, _ = O.tfs_aggregate(row, col, xq, wq, L, R, K, d, mx=mx, rounding=O.TFS_EDGE)
    close(out, t["b1_out_" + key], 5e-5)
    assert np.array_equal(den, t["b1_den_" + key])
    for name, rounding, block, thr in (("online16", O.TFS_EDGE, 16, 1), ("block32", O.TFS_BLOCK, 32, 1),
                                       ("hybrid32", O.TFS_SPLIT if (K, d) == (8, 32) else O.TFS_BLOCK, 32, 16)):
        out, den, m = O.tfs_aggregate(row, col, xq, wq, L, R, K, d, rounding=rounding, block=block, threshold=thr)
        close(out, t[f"{name}_out_{key}"], 2e-4 if name == "hybrid32" else 5e-5)
        assert np.array_equal(den, t[f"{name}_den_{key}"]), name
        assert np.array_equal(m, t[f"{name}_max_{key}"]), name
        # the running maximum ends at the prescan maximum (leaky is monotone)
        nz = np.diff(row.astype(np.int64)) > 0
        assert np.array_equal(m[nz], mx[nz])


@pytest.mark.parametrize("name", ["smoke1024_seed11", "config1"])
def test_tfs_chain_matches_reference(name):
    """Three tfs_layer calls (path tfs_bf16, lr policy bf16) vs the reference."""
    import configs
    g = np.load(GOLDEN / f"{name}.npz")
    if name == "config1":
        cfg = configs.make("c1")
        graph, model = cfg.graph, [(p.w, p.al, p.ar, p.heads, p.dim) for p in cfg.model]
    else:
        graph, model = smoke1024_graph(), O.random_model(128, 40, 11)
    inp = graph.x
    for l, (w, al, ar, h, d) in enumerate(model):
        inp = O.tfs_layer(graph.row, graph.col, inp, w, al, ar, h, d, l < 2)
    e = O.errors(g["tfsbf16_logits"], inp)
    # L/R come from a BF16 GEMM whose summation order differs from oneMKL's;
    # every layer re-rounds to BF16, so last-bit differences flip some
    # roundings (as for the B0 chain).
    assert e["relative_l2"] <= 5e-4, e
    r0 = O.errors(g["ref_logits"], inp)
    assert r0["relative_l2"] <= 2e-2, r0  # TFS BF16 vs R0: same order as B0 BF16


def _fixture_inputs():
    import gatb200 as G
    g = G.load_graph(GOLDEN / "fixture_small.gatbin")
    assert hashlib.sha256((GOLDEN / "fixture_small.gatbin").read_bytes()).hexdigest() == MANIFEST[
        "fixture_small_gatbin_sha256"]
    return g, G.random_model(g.din, g.classes, 11)


def test_reference_fixture_round_trip(tmp_path):
    """The reference's export-fixture file (GATFIX1, common.cpp:171-194) reads and
    validates, holds the R0 weights of layer 1, and our writer reproduces it byte
    for byte."""
    import gatb200 as G
    g, model = _fixture_inputs()
    p = model[0]
    path = GOLDEN / "fixture_small_l1.gatfix"
    x, pw, den = G.read_fixture(path, g.row, g.col, p)
    assert np.array_equal(x, g.x)  # layer 1 input is the graph's features
    o = O.ref_layer(g.row, g.col, x, p.w, p.al, p.ar, p.heads, p.dim, False, want_p=True)
    assert np.abs(pw - o["p"]).max() <= 1e-6 and np.abs(den - o["den"]).max() <= 1e-5 * np.abs(den).max()
    G.write_fixture(tmp_path / "again.gatfix", g.row, g.col, p, x, pw, den)
    assert (tmp_path / "again.gatfix").read_bytes() == path.read_bytes()


def test_fixture_validation_messages(tmp_path):
    """load_fixture's checks (common.cpp:181-193) with the reference's messages."""
    import gatb200 as G
    g, model = _fixture_inputs()
    p = model[0]
    x, pw, den = G.read_fixture(GOLDEN / "fixture_small_l1.gatfix", g.row, g.col, p)

    def expect(msg, path, row=g.row, col=g.col, layer=p):
        with pytest.raises(RuntimeError, match=msg):
            G.read_fixture(path, row, col, layer)

    bad = tmp_path / "bad.gatfix"
    raw = bytearray((GOLDEN / "fixture_small_l1.gatfix").read_bytes())
    raw[0] = ord("X")
    bad.write_bytes(bytes(raw))
    expect("bad fixture magic", bad)
    expect("fixture shape mismatch", GOLDEN / "fixture_small_l1.gatfix", layer=model[1])
    col2 = g.col.copy()
    col2[5] = (col2[5] + 1) % g.n
    expect("fixture CSR mismatch", GOLDEN / "fixture_small_l1.gatfix", col=col2)
    w2 = p.w.copy()
    w2[0, 0] += 1.0
    expect("fixture checkpoint mismatch", GOLDEN / "fixture_small_l1.gatfix",
           layer=G.Param(p.in_, p.heads, p.dim, w2, p.al, p.ar))
    p2 = pw.copy()
    p2[3, 0] = 1.5
    G.write_fixture(bad, g.row, g.col, p, x, p2, den)
    expect("fixture p outside", bad)
    d2 = den.copy()
    d2[4, 1] *= 1.01
    G.write_fixture(bad, g.row, g.col, p, x, pw, d2)
    expect("fixture denominator mismatch", bad)


@pytest.mark.parametrize("block", [4, 16, 64])
def test_online_counters_match_reference(golden, block):
    """icpp_online's exact counters (icpp_online.hpp:18-22) from the reference
    (ref_dump counters, smoke1024, scores rising with the source id): per (row,
    head) blocks, max updates and rescales, and the Stats totals, bit-exact.
    The derived totals follow from them as the reference computes them."""
    g = smoke1024_graph()
    c = np.load(golden / "tfs_counters.npz")
    perm, _ = O.degree_schedule(g.row)
    rb, ru, rr, tot = O.online_counters(g.row, g.col, perm, c["left"], c["right"], 8, block)
    assert np.array_equal(rb, c[f"rowblocks_b{block}"])
    assert np.array_equal(ru, c[f"rowupdates_b{block}"])
    assert np.array_equal(rr, c[f"rowrescales_b{block}"])
    want = c[f"totals_b{block}"]
    assert np.array_equal(tot, want[:5])
    # amx_calls, executed_fma, rescaled (padded) feature elements, spill/reload bytes
    dp, obs, d = 128, 2, 32  # padded_in of D=128, output blocks of d=32
    steps, rescales, events = int(tot[4]), int(tot[2]), int(tot[3])
    assert int(want[5]) == steps * (dp // 32) * obs
    assert int(want[6]) == steps * 16 * dp * obs * 16
    assert int(want[7]) == rescales * d and int(want[8]) == rescales * obs * 16
    assert int(want[9]) == int(want[10]) == events * obs * 1024
    assert rescales > 0 and events > 0  # the case exercises rescaling
