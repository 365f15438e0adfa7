"""Parity of the TFS path (lr_reordered, TFS aggregation, tfs_layer, the
TFS_BF16 and ADAPTIVE_BF16 model paths) with the CPU oracle, through the C-ABI.

Tolerances:
  * lr_reordered: bit-exact (the kernel runs the oracle's FMA chain on the
    same blr; BF16 copy of X bit-exact);
  * TFS aggregation: the CUDA-core kernel runs the restatement's arithmetic
    in the same order, so outputs differ only through expf (CUDA vs glibc,
    <= 2 ulp of p). Every variant rounds to BF16 downstream of p (p*x for
    EDGE, U for BLOCK/SPLIT, p itself for SPLIT's high/low parts), and an ulp
    of p can flip one such rounding, moving one term by a BF16 step (2^-8
    relative): relative L2 <= 1e-4 and max-abs <= 1e-3 x scale; den to 1e-6
    relative. With caller weights (fixed_p) there is no expf, and the output
    is bit-exact: that pins the order of the arithmetic;
  * against the reference's own outputs (tests/golden/tfs.npz) the oracle's
    pin tolerances apply (AMX accumulation order): 5e-5 / 2e-4 x scale;
  * model paths: relative L2 <= 1e-2 against R0 (north-star BF16 gate).
"""
import numpy as np
import pytest

import gatb200 as G
import oracle as O
from test_gpu_parity import T, host, hub_graph, rel_l2, random_layer

pytestmark = pytest.mark.gpu

TFS_CASES = [(17, 1, 7), (33, 2, 40), (128, 8, 32), (256, 8, 32), (256, 1, 47), (128, 4, 47)]


def _close(got, want, rel, what=""):
    scale = max(1e-30, float(np.abs(want).max()))
    err = float(np.abs(got - want).max()) / scale
    assert err <= rel, (what, err)


def _close_exp(got, want, what=""):
    """Same arithmetic, weights from two expf implementations (see module doc)."""
    _close(got, want, 1e-3, what)
    assert rel_l2(want, got) <= 1e-4, (what, rel_l2(want, got))


def _bf16_table(x, ld):
    b = np.zeros((x.shape[0], ld), np.uint16)
    b[:, : x.shape[1]] = G.rne(x)
    return b


def _run_tfs(g, layer, xtab, ld, L, R, n, K, d, mx=None, rounding=G.TFS_EDGE, block=0, threshold=1, fixed_p=None,
             fixed_den=None, want_max=False):
    import torch
    out = torch.full((n, K * d), float("nan"), dtype=torch.float32, device="cuda")
    den = torch.full((n, K), float("nan"), dtype=torch.float32, device="cuda")
    mo = torch.full((n, K), float("nan"), dtype=torch.float32, device="cuda") if want_max else None
    G.tfs_aggregate(g, layer, T(xtab.view(np.int16)), ld, None if L is None else T(L), None if R is None else T(R),
                    out, K * d, den, mx=None if mx is None else T(mx), rounding=rounding, block=block,
                    threshold=threshold, fixed_p=None if fixed_p is None else T(fixed_p),
                    fixed_den=None if fixed_den is None else T(fixed_den), max_out=mo)
    return host(out), host(den), (host(mo) if want_max else None)


@pytest.mark.parametrize("D", [17, 33, 100, 128, 256])
@pytest.mark.parametrize("policy", [G.LR_BF16, G.LR_FP32])
def test_lr_reordered_bit_exact(dev, D, policy):
    import torch
    rng = np.random.default_rng(D)
    for K, d in ((8, 32), (1, 47), (2, 7)):
        p = random_layer(rng, D, K, d)
        layer = G.DeviceLayer(p)
        n = 1000
        x = rng.standard_normal((n, D)).astype(np.float32)
        ldb = G.padded_ld(D, G.BF16)
        left = torch.empty((n, K), dtype=torch.float32, device="cuda")
        right = torch.empty((n, K), dtype=torch.float32, device="cuda")
        xb = torch.full((n, ldb), -1, dtype=torch.int16, device="cuda")
        G.lr_reordered(layer, n, T(x), G.F32, D, policy, left, right, x_bf16=xb, ld_bf16=ldb)
        blr = O.prepare_blr(p.w, p.al, p.ar, K, d)
        wl, wr = O.lr_reordered(x, blr, K, policy)
        assert np.array_equal(host(left), wl) and np.array_equal(host(right), wr), (D, K, d)
        assert np.array_equal(host(xb), _bf16_table(x, ldb))
        # BF16 input (layers 2-3 of the TFS path): only the bf16 policy reads X in BF16
        if policy == G.LR_BF16:
            G.lr_reordered(layer, n, xb, G.BF16, ldb, policy, left, right)
            assert np.array_equal(host(left), wl) and np.array_equal(host(right), wr)
        layer.close()


@pytest.mark.parametrize("case", TFS_CASES, ids=lambda c: "_".join(map(str, c)))
def test_tfs_aggregate_variants(dev, golden, case):
    D, K, d = case
    key = f"{D}_{K}_{d}"
    t = np.load(golden / "tfs.npz")
    row, col, x = O.boundary_graph(D)
    w, al, ar = O.boundary_params(D, K, d)
    layer = G.DeviceLayer(G.Param(D, K, d, w, al, ar))
    g = G.DeviceGraph(row, col)
    n = 35
    ld = G.padded_ld(D, G.BF16)
    xtab = _bf16_table(x, ld)
    xq, wq = O.quantize(x), O.quantize(w)
    L, R, mx = t["lbf_" + key], t["rbf_" + key], t["max_" + key]
    # B1 (tfs_aggregate with the prescan max)
    out, den, _ = _run_tfs(g, layer, xtab, ld, L, R, n, K, d, mx=mx)
    oo, od, _ = O.tfs_aggregate(row, col, xq, wq, L, R, K, d, mx=mx, rounding=O.TFS_EDGE)
    _close_exp(out, oo, "b1 vs oracle")
    _close(den, od, 1e-6, "b1 den")
    _close_exp(out, t["b1_out_" + key], "b1 vs reference")
    # online / block / split (running max per block)
    for name, rounding, block, thr in (("online16", G.TFS_EDGE, 16, 1), ("block32", G.TFS_BLOCK, 32, 1),
                                       ("hybrid32", G.TFS_SPLIT, 32, 16)):
        out, den, m = _run_tfs(g, layer, xtab, ld, L, R, n, K, d, rounding=rounding, block=block, threshold=thr,
                               want_max=True)
        oo, od, om = O.tfs_aggregate(row, col, xq, wq, L, R, K, d, rounding=rounding, block=block, threshold=thr)
        _close_exp(out, oo, name)
        _close(den, od, 1e-6, name + " den")
        assert np.array_equal(m, om), name
        if name != "hybrid32" or (K, d) == (8, 32):  # the reference splits p only for K8 d32
            _close_exp(out, t[f"{name}_out_{key}"], name + " vs reference")
    # the B200 semantics: SPLIT, one block per row, prescan maximum
    # (rows longer than the graph's segment length take one block per segment)
    out, den, _ = _run_tfs(g, layer, xtab, ld, L, R, n, K, d, mx=mx, rounding=G.TFS_SPLIT, block=0)
    oo, od, _ = O.tfs_aggregate(row, col, xq, wq, L, R, K, d, mx=mx, rounding=O.TFS_SPLIT,
                                block=g.info()["seg_edges"])
    _close_exp(out, oo, "split block 0")
    _close(den, od, 1e-6, "split block 0 den")
    # empty rows: zero output and den (baseline_tfs.cpp:89-91)
    assert np.all(out[0] == 0) and np.all(den[0] == 0)
    layer.close()
    g.close()


def test_tfs_fixed_p(dev):
    """B1 fixed-p mode (bench/main.cpp:133): weights and den from the caller."""
    rng = np.random.default_rng(3)
    row, col = hub_graph(n=600, hubs=(500, 300), seed=2)
    n, e = len(row) - 1, len(col)
    K, d, D = 8, 32, 64
    p = random_layer(rng, D, K, d)
    layer = G.DeviceLayer(p)
    g = G.DeviceGraph(row, col)
    x = rng.standard_normal((n, D)).astype(np.float32)
    ld = G.padded_ld(D, G.BF16)
    fp = rng.uniform(0, 1, (e, K)).astype(np.float32)
    fd = rng.uniform(1, 2, (n, K)).astype(np.float32)
    out, den, _ = _run_tfs(g, layer, _bf16_table(x, ld), ld, None, None, n, K, d, fixed_p=fp, fixed_den=fd)
    oo, od, _ = O.tfs_aggregate(row, col, O.quantize(x), O.quantize(p.w), None, None, K, d, fixed_p=fp, fixed_den=fd)
    # identical weights: the only difference left is none (same order, same products)
    assert np.array_equal(out, oo)
    assert np.array_equal(den, fd)
    layer.close()
    g.close()


@pytest.mark.parametrize("rounding,block", [(G.TFS_EDGE, 0), (G.TFS_SPLIT, 0), (G.TFS_BLOCK, 32)])
def test_tfs_hub_rows(dev, rounding, block):
    """Rows far longer than a block or segment (the tensor-core kernel splits them)."""
    import torch
    rng = np.random.default_rng(11)
    row, col = hub_graph(n=3000, seed=9)
    n = len(row) - 1
    K, d, D = 8, 32, 100
    p = random_layer(rng, D, K, d)
    layer = G.DeviceLayer(p)
    g = G.DeviceGraph(row, col)
    x = rng.standard_normal((n, D)).astype(np.float32)
    ld = G.padded_ld(D, G.BF16)
    L = (rng.standard_normal((n, K)) * 0.5).astype(np.float32)
    R = (rng.standard_normal((n, K)) * 0.5).astype(np.float32)
    mx = O.max_prescan(row, col, L, R, K)
    use_max = block == 0
    out, den, _ = _run_tfs(g, layer, _bf16_table(x, ld), ld, L, R, n, K, d, mx=mx if use_max else None,
                           rounding=rounding, block=block)
    info = g.info()
    assert info["n_hub"] > 0
    # block 0 with BLOCK/SPLIT rounding: one block per row, one per segment of
    # seg_edges for the rows longer than that
    ob = block if block else (info["seg_edges"] if rounding != G.TFS_EDGE else 0)
    oo, od, _ = O.tfs_aggregate(row, col, O.quantize(x), O.quantize(p.w), L, R, K, d, mx=mx if use_max else None,
                                rounding=rounding, block=ob)
    _close_exp(out, oo, "hubs")
    _close(den, od, 1e-5, "hubs den")
    layer.close()
    g.close()


def _tfs_chain_oracle(graph, params, rounding=O.TFS_EDGE):
    inp = graph.x
    for l, p in enumerate(params):
        inp = O.tfs_layer(graph.row, graph.col, inp, p.w, p.al, p.ar, p.heads, p.dim, l < 2, rounding=rounding)
    return inp


def test_tfs_layer_entry_point(dev):
    import torch
    import configs
    cfg = configs.make("c1")
    gr, p = cfg.graph, cfg.model[0]
    g = G.DeviceGraph(gr.row, gr.col)
    layer = G.DeviceLayer(p)
    n = gr.n
    ldb = G.padded_ld(p.in_, G.BF16)
    f32 = dict(dtype=torch.float32, device="cuda")
    xb = torch.zeros((n, ldb), dtype=torch.int16, device="cuda")
    left, right, mx, den = (torch.empty((n, p.heads), **f32) for _ in range(4))
    out = torch.empty((n, p.width), **f32)
    G.tfs_layer(g, layer, T(gr.x), G.F32, p.in_, True, xb, left, right, mx, den, out, G.F32, p.width)
    want = O.tfs_layer(gr.row, gr.col, gr.x, p.w, p.al, p.ar, p.heads, p.dim, True)
    _close_exp(host(out), want, "tfs_layer")
    layer.close()
    g.close()


@pytest.mark.parametrize("name", ["config1", "smoke1024_seed11"])
def test_tfs_model_paths(dev, golden, name):
    import configs
    from test_gpu_parity import _model, _forward, _smoke_inputs
    ref = np.load(golden / f"{name}.npz")
    if name == "config1":
        cfg = configs.make("c1")
        graph, params = cfg.graph, cfg.model
    else:
        graph, params = _smoke_inputs(golden), G.random_model(128, 40, 11)
    # path tfs_bf16 (B1 on every layer) against the reference's own tfs_bf16 chain
    _, _, mt = _model(graph, params, G.PATH_TFS_BF16)
    got = _forward(mt, graph.x)
    assert rel_l2(ref["tfsbf16_logits"], got) <= 1e-3
    assert rel_l2(_tfs_chain_oracle(graph, params), got) <= 5e-4
    assert rel_l2(ref["ref_logits"], got) <= 1e-2
    # adaptive: layer 1 TFS (SPLIT, one block per row), layers 2-3 B0 BF16
    _, _, ma = _model(graph, params, G.PATH_ADAPTIVE_BF16)
    got_a = _forward(ma, graph.x)
    assert rel_l2(ref["ref_logits"], got_a) <= 1e-2
    p0 = params[0]
    inp = O.tfs_layer(graph.row, graph.col, graph.x, p0.w, p0.al, p0.ar, p0.heads, p0.dim, True,
                      rounding=O.TFS_SPLIT)
    for l, p in enumerate(params[1:], 1):
        inp = O.b0_layer(graph.row, graph.col, inp, p.w, p.al, p.ar, p.heads, p.dim, l < 2, bf16=True,
                         round_z=True)["out"]
    assert rel_l2(inp, got_a) <= 3e-3


def test_adaptive_model_tensor_core_layer(dev):
    """Adaptive path with a layer-1 shape the tcgen05 TFS kernel takes (in=100):
    power-law degrees with hub rows split into segments, against the oracle
    (layer 1 TFS with heads_hybrid rounding, one block per row or segment;
    layers 2-3 B0 BF16 with H rounded to BF16 as the device stores it)."""
    from test_gpu_parity import _model, _forward
    n, e = 20000, 420000
    row, col = G.synth_powerlaw_graph(n, e, 6000, 2.1, 17)
    x = G.synth_normal((n, 100), 17, 1)
    params = G.glorot_model(100, 47, 17)
    graph = G.Graph(n=n, e=e, din=100, classes=47, row=row, col=col, x=x)
    g, _, m = _model(graph, params, G.PATH_ADAPTIVE_BF16)
    info = g.info()
    assert info["n_hub"] > 0
    got = _forward(m, x)
    p0 = params[0]
    blr = O.prepare_blr(p0.w, p0.al, p0.ar, p0.heads, p0.dim)
    L, R = O.lr_reordered(x, blr, p0.heads, 0)
    mx = O.max_prescan(row, col, L, R, p0.heads)
    out, den, _ = O.tfs_aggregate(row, col, O.quantize(x), O.quantize(p0.w), L, R, p0.heads, p0.dim, mx=mx,
                                  rounding=O.TFS_SPLIT, block=info["seg_edges"])
    inp = O.finish(out, den, p0.heads, p0.dim, True)
    for l, p in enumerate(params[1:], 1):
        inp = O.b0_layer(row, col, inp, p.w, p.al, p.ar, p.heads, p.dim, l < 2, bf16=True, round_z=True)["out"]
    assert rel_l2(inp, got) <= 3e-3
    ref = O.ref_chain(row, col, x, [(p.w, p.al, p.ar, p.heads, p.dim) for p in params])[2]["out"]
    assert rel_l2(ref, got) <= 1e-2


def test_reference_fixture_fixed_p(dev, golden):
    """Fixed-p mode on the reference's own GATFIX1 fixture (bench/main.cpp:127-138):
    the standard path (BF16 projection, aggregation with the fixture's p and den,
    finish) and the TFS B1 path with the same weights."""
    import torch
    g_host = G.load_graph(golden / "fixture_small.gatbin")
    params = G.random_model(g_host.din, g_host.classes, 11)
    p = params[0]
    x, pw, den = G.read_fixture(golden / "fixture_small_l1.gatfix", g_host.row, g_host.col, p)
    n, K, d, W = g_host.n, p.heads, p.dim, p.width
    g = G.DeviceGraph(g_host.row, g_host.col)
    layer = G.DeviceLayer(p)
    ld = G.padded_ld(p.in_, G.BF16)
    xb = T(_bf16_table(x, ld).view(np.int16))
    f32 = dict(dtype=torch.float32, device="cuda")
    # standard fixed-p
    ldh = G.padded_ld(W, G.BF16)
    h = torch.zeros((n, ldh), dtype=torch.int16, device="cuda")
    lft, rgt = torch.empty((n, K), **f32), torch.empty((n, K), **f32)
    G.projection(layer, n, xb, ld, G.BF16, h, G.BF16, ldh, lft, rgt)
    out = torch.empty((n, W), **f32)
    dn = torch.empty((n, K), **f32)
    G.standard_aggregate(g, K, d, h, G.BF16, ldh, lft, rgt, out, W, dn, fixed_p=T(pw), fixed_den=T(den))
    G.finish(n, K, d, dn, False, out, W)
    z = O.quantize(O.quantize(x) @ O.quantize(p.w))  # BF16 X . BF16 W, H stored in BF16
    so, sd = O.standard_aggregate(g_host.row, g_host.col, z, None, None, None, K, d, fixed_p=pw, fixed_den=den)
    want = O.finish(so, sd, K, d, False)
    assert np.array_equal(host(dn), den)
    assert rel_l2(want, host(out)) <= 1e-3
    # TFS B1 fixed-p: same weights, same arithmetic order as the oracle -> bit-exact
    out2, den2, _ = _run_tfs(g, layer, _bf16_table(x, ld), ld, None, None, n, K, d, fixed_p=pw, fixed_den=den)
    oo, od, _ = O.tfs_aggregate(g_host.row, g_host.col, O.quantize(x), O.quantize(p.w), None, None, K, d,
                                fixed_p=pw, fixed_den=den)
    assert np.array_equal(out2, oo) and np.array_equal(den2, den)
    # and the two paths agree as the reference's fixed-p control reports (extra pX rounding only)
    assert rel_l2(O.finish(oo, od, K, d, False), host(out)) <= 1e-2
    layer.close()
    g.close()


def test_matched_attention_model(dev, golden):
    """matched_attention (bench/main.cpp:22-25): B0 BF16 with L/R from lr_reordered."""
    import configs
    from test_gpu_parity import _model, _forward
    ref = np.load(golden / "config1.npz")
    cfg = configs.make("c1")
    graph, params = cfg.graph, cfg.model
    _, _, m = _model(graph, params, G.PATH_MATCHED_ATTENTION)
    got = _forward(m, graph.x)
    inp = graph.x
    for l, p in enumerate(params):
        xq = O.quantize(inp)
        z = O.quantize(xq @ O.quantize(p.w))  # H stored in BF16 as the device does
        blr = O.prepare_blr(p.w, p.al, p.ar, p.heads, p.dim)
        L, R = O.lr_reordered(inp, blr, p.heads, 0)
        mx = O.max_prescan(graph.row, graph.col, L, R, p.heads)
        out, den = O.standard_aggregate(graph.row, graph.col, z, L, R, mx, p.heads, p.dim)
        inp = O.finish(out, den, p.heads, p.dim, l < 2)
    assert rel_l2(inp, got) <= 3e-3
    assert rel_l2(ref["ref_logits"], got) <= 1e-2


@pytest.mark.parametrize("block", [4, 16, 64])
def test_online_counters_match_reference(dev, golden, block):
    """gat_b200_tfs_online_counters against the reference's own icpp_online
    counters (ref_dump counters on smoke1024; tests/golden/tfs_counters.npz):
    per (row, head) blocks / max updates / rescales and the totals, bit-exact."""
    import torch
    from test_oracle_golden import smoke1024_graph
    g = smoke1024_graph()
    c = np.load(golden / "tfs_counters.npz")
    dg = G.DeviceGraph(g.row, g.col)
    n = g.n
    bufs = [torch.zeros((n, 8), dtype=torch.int64, device="cuda") for _ in range(3)]
    tot = G.tfs_online_counters(dg, 8, T(c["left"]), T(c["right"]), block, *bufs)
    for buf, name in zip(bufs, ("rowblocks", "rowupdates", "rowrescales")):
        assert np.array_equal(host(buf).astype(np.uint64), c[f"{name}_b{block}"]), name
    assert np.array_equal(tot, c[f"totals_b{block}"][:5])
    dg.close()


@pytest.mark.parametrize("block", [3, 32])
def test_online_counters_match_oracle_on_hubs(dev, block):
    """Same counters on the hub graph (rows far above the segment length) against
    the oracle restatement."""
    import torch
    row, col = hub_graph()
    n = len(row) - 1
    rng = np.random.default_rng(block)
    K = 4
    left = rng.standard_normal((n, K)).astype(np.float32)
    right = (rng.standard_normal((n, K)) + np.arange(n)[:, None] * 1e-3).astype(np.float32)
    dg = G.DeviceGraph(row, col)
    bufs = [torch.zeros((n, K), dtype=torch.int64, device="cuda") for _ in range(3)]
    tot = G.tfs_online_counters(dg, K, T(left), T(right), block, *bufs)
    perm, _ = O.degree_schedule(row)
    rb, ru, rr, otot = O.online_counters(row, col, perm, left, right, K, block)
    for buf, want in zip(bufs, (rb, ru, rr)):
        assert np.array_equal(host(buf).astype(np.uint64), want)
    assert np.array_equal(tot, otot)
    assert otot[2] > 0
    dg.close()


@pytest.mark.parametrize("block", [16, 32, 64])
def test_online_equals_b1_when_scores_are_equal(dev, block):
    """The reference's all-equal-scores lifecycle check (tfs_online/checks.cpp:452-520):
    with every score equal the running maximum never rises after a row's first block, so
    the online variant takes the same weights as B1 with the prescan maximum, bit for bit;
    the counters show no rescale."""
    import torch
    rng = np.random.default_rng(block)
    row, col = hub_graph(n=600, hubs=(500, 300), seed=4)
    n = len(row) - 1
    K, d, D = 8, 32, 64
    p = random_layer(rng, D, K, d)
    layer = G.DeviceLayer(p)
    g = G.DeviceGraph(row, col)
    x = rng.standard_normal((n, D)).astype(np.float32)
    ld = G.padded_ld(D, G.BF16)
    L = np.full((n, K), 0.25, np.float32)
    R = np.full((n, K), -0.75, np.float32)
    mx = O.max_prescan(row, col, L, R, K)
    b1, b1d, _ = _run_tfs(g, layer, _bf16_table(x, ld), ld, L, R, n, K, d, mx=mx)
    on, ond, _ = _run_tfs(g, layer, _bf16_table(x, ld), ld, L, R, n, K, d, block=block)
    assert np.array_equal(on, b1) and np.array_equal(ond, b1d)
    tot = G.tfs_online_counters(g, K, T(L), T(R), block)
    assert int(tot[2]) == 0 and int(tot[3]) == 0
    layer.close()
    g.close()
