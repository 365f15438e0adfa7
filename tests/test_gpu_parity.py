"""Parity of the CUDA path (through the C-ABI) with the CPU oracle.

Every call goes through libgat_b200.so; device buffers are torch tensors used
only as memory. Tolerances:
  * integer / index work (degree schedule, row max): bit-exact;
  * FP32 path: max-abs <= 1e-5 against the R0 oracle (north-star gate);
  * BF16 path: relative L2 <= 1e-2 against R0 (north-star gate), and tighter
    checks against the B0 restatement that rounds the same intermediates.
"""
import numpy as np
import pytest

import gatb200 as G
import oracle as O

pytestmark = pytest.mark.gpu


def T(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def dev_bf16(x: np.ndarray, ld: int):
    """BF16 RNE copy of FP32 rows with a padded stride (padding zero)."""
    import torch
    n, w = x.shape
    b = np.zeros((n, ld), np.uint16)
    b[:, :w] = G.rne(x)
    return torch.from_numpy(b.view(np.int16)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    G.check_device()
    a = t.cpu().numpy()
    return a.view(np.uint16) if a.dtype == np.int16 else a


def rel_l2(ref, got):
    return O.errors(ref, got)["relative_l2"]


def random_layer(rng, D, K, d, scale=None):
    s = scale or 1.0 / np.sqrt(D)
    w = (rng.standard_normal((D, K * d)) * s).astype(np.float32)
    al = (rng.standard_normal(K * d) / np.sqrt(d)).astype(np.float32)
    ar = (rng.standard_normal(K * d) / np.sqrt(d)).astype(np.float32)
    return G.Param(D, K, d, w, al, ar)


def hub_graph(n=3000, hubs=(2900, 2500, 1800, 700), seed=5):
    """Mostly tiny rows plus a few rows far above the segment length."""
    rng = np.random.default_rng(seed)
    row, col = [0], []
    for i in range(n):
        deg = hubs[i % len(hubs)] if i % 500 == 7 else int(rng.integers(0, 6))
        col.extend(sorted(rng.choice(n, size=deg, replace=False).tolist()))
        row.append(len(col))
    return np.array(row, np.uint64), np.array(col, np.uint32)


# ------------------------------------------------------------ degree schedule
def test_degree_schedule_bit_exact(dev, golden):
    import configs
    b = np.load(golden / "boundary.npz")
    cases = [(b["row"], b["col"])]
    c1 = configs.make("c1", features=False).graph
    cases.append((c1.row, c1.col))
    c2 = configs.make_graph("c2", features=False)
    cases.append((c2.row, c2.col))
    cases.append(hub_graph())
    for row, col in cases:
        g = G.DeviceGraph(row, col)
        perm, steps = g.schedule()
        operm, osteps = O.degree_schedule(row)
        assert np.array_equal(perm, operm)
        assert steps == osteps
    # the reference's own perm for its boundary graph
    g = G.DeviceGraph(b["row"], b["col"])
    perm, steps = g.schedule()
    assert np.array_equal(perm, b["perm"]) and steps == int(b["steps"][0])


def test_device_graph_validation_messages(dev):
    row = np.array([0, 2, 3, 3, 6], np.uint64)
    col = np.array([1, 2, 0, 0, 1, 3], np.uint32)
    bad = row.copy()
    bad[2] = 7
    with pytest.raises(G.GatError, match="nonmonotone CSR"):
        G.DeviceGraph(bad, col)
    badc = col.copy()
    badc[3] = 9
    with pytest.raises(G.GatError, match="source index out of bounds"):
        G.DeviceGraph(row, badc)
    badb = row.copy()
    badb[0] = 1
    with pytest.raises(G.GatError, match="bad CSR bounds"):
        G.DeviceGraph(badb, col)


# ------------------------------------------------------------ projection
PROJ_SHAPES = [(35, 17, 1, 7), (35, 256, 8, 32), (1000, 100, 8, 32), (5000, 256, 8, 32), (4097, 256, 1, 47),
               (300, 33, 2, 40), (129, 128, 4, 47), (200, 17, 8, 47), (777, 256, 1, 40), (260, 64, 1, 64)]


@pytest.mark.parametrize("n,D,K,d", PROJ_SHAPES)
def test_projection_bf16(dev, n, D, K, d):
    import torch
    rng = np.random.default_rng(n + D + K + d)
    x = rng.standard_normal((n, D)).astype(np.float32)
    p = random_layer(rng, D, K, d)
    layer = G.DeviceLayer(p)
    ldx, W = G.padded_ld(D, G.BF16), K * d
    xb = dev_bf16(x, ldx)
    ldh = G.padded_ld(W, G.BF16)
    h = torch.full((n, ldh), -1, dtype=torch.int16, device="cuda")
    left = torch.empty((n, K), dtype=torch.float32, device="cuda")
    right = torch.empty((n, K), dtype=torch.float32, device="cuda")
    G.projection(layer, n, xb, ldx, G.BF16, h, G.BF16, ldh, left, right)
    z64 = O.quantize(x).astype(np.float64) @ O.quantize(p.w).astype(np.float64)
    H = G.bf16_to_f32(host(h)[:, :W]).astype(np.float64)
    assert np.all(np.abs(H - z64) <= 2.0 ** -8 * np.abs(z64) + 1e-5)
    assert np.all(host(h)[:, W:] == 0), "padding columns must be zero"
    zh = z64.reshape(n, K, d)
    L = np.einsum("nhd,hd->nh", zh, p.al.reshape(K, d).astype(np.float64))
    R = np.einsum("nhd,hd->nh", zh, p.ar.reshape(K, d).astype(np.float64))
    assert np.abs(host(left) - L).max() <= 1e-5 * max(1, np.abs(L).max())
    assert np.abs(host(right) - R).max() <= 1e-5 * max(1, np.abs(R).max())
    # FP32 Z output (the reference's projection() result) through the same kernel
    ld32 = G.padded_ld(W, G.F32)
    z32 = torch.empty((n, ld32), dtype=torch.float32, device="cuda")
    G.projection(layer, n, xb, ldx, G.BF16, z32, G.F32, ld32, None, None)
    assert np.abs(host(z32)[:, :W] - z64).max() <= 1e-5 * max(1, np.abs(z64).max())


@pytest.mark.parametrize("n,D,K,d", [(35, 17, 1, 7), (1000, 100, 8, 32), (300, 33, 2, 40), (200, 17, 8, 47)])
def test_projection_fp32(dev, n, D, K, d):
    import torch
    rng = np.random.default_rng(7 * n + D)
    x = rng.standard_normal((n, D)).astype(np.float32)
    p = random_layer(rng, D, K, d)
    layer = G.DeviceLayer(p)
    W = K * d
    ld = G.padded_ld(W, G.F32)
    h = torch.empty((n, ld), dtype=torch.float32, device="cuda")
    left = torch.empty((n, K), dtype=torch.float32, device="cuda")
    right = torch.empty((n, K), dtype=torch.float32, device="cuda")
    G.projection(layer, n, T(x), D, G.F32, h, G.F32, ld, left, right)
    row = np.zeros(n + 1, np.uint64)
    o = O.ref_layer(row, np.zeros(0, np.uint32), x, p.w, p.al, p.ar, K, d, False)
    assert np.abs(host(h)[:, :W] - o["z"]).max() <= 1e-5 * max(1, np.abs(o["z"]).max())
    assert np.abs(host(left) - o["left"]).max() <= 1e-5 * max(1, np.abs(o["left"]).max())
    assert np.abs(host(right) - o["right"]).max() <= 1e-5 * max(1, np.abs(o["right"]).max())


# ------------------------------------------------------------ aggregation
def _agg_case(row, col, n, K, d, seed, dtype):
    import torch
    rng = np.random.default_rng(seed)
    z = rng.standard_normal((n, K * d)).astype(np.float32)
    if dtype == G.BF16:
        z = O.quantize(z)
    left = rng.standard_normal((n, K)).astype(np.float32)
    right = rng.standard_normal((n, K)).astype(np.float32)
    ld = G.padded_ld(K * d, dtype)
    if dtype == G.BF16:
        h = dev_bf16(z, ld)
    else:
        hz = np.zeros((n, ld), np.float32)
        hz[:, :K * d] = z
        h = T(hz)
    return z, left, right, h, ld


AGG_SHAPES = [(1, 7), (2, 32), (4, 40), (8, 32), (8, 47), (1, 47), (1, 64), (2, 7)]


@pytest.mark.parametrize("K,d", AGG_SHAPES)
@pytest.mark.parametrize("dtype", [G.F32, G.BF16])
@pytest.mark.parametrize("graph", ["boundary", "hubs"])
def test_standard_aggregate(dev, golden, K, d, dtype, graph):
    import torch
    if graph == "boundary":
        b = np.load(golden / "boundary.npz")
        row, col = b["row"], b["col"]
    else:
        row, col = hub_graph()
    n = len(row) - 1
    z, left, right, h, ld = _agg_case(row, col, n, K, d, K * 100 + d, dtype)
    g = G.DeviceGraph(row, col)
    W = K * d
    out = torch.full((n, W), 7.0, dtype=torch.float32, device="cuda")
    den = torch.empty((n, K), dtype=torch.float32, device="cuda")
    mx = torch.empty((n, K), dtype=torch.float32, device="cuda")
    G.standard_aggregate(g, K, d, h, dtype, ld, T(left), T(right), out, W, den, mx)
    omax = O.max_prescan(row, col, left, right, K)
    oout, oden = O.standard_aggregate(row, col, z, left, right, omax, K, d)
    assert np.array_equal(host(mx), omax), "row max must be bit-exact"
    assert np.abs(host(den) - oden).max() <= 1e-5 * max(1, np.abs(oden).max())
    assert np.abs(host(out) - oout).max() <= 1e-5 * max(1, np.abs(oout).max())
    # max_prescan kernel alone (baseline_standard.cpp:44-51)
    m2 = torch.empty((n, K), dtype=torch.float32, device="cuda")
    G.max_prescan(g, K, T(left), T(right), m2)
    assert np.array_equal(host(m2), omax)
    # finish (normalise + ELU), then the fused kernel must equal both steps
    G.finish(n, K, d, den, True, out, W)
    fin = O.finish(oout, oden, K, d, True)
    assert np.abs(host(out) - fin).max() <= 1e-5
    fused = torch.empty((n, W), dtype=torch.float32, device="cuda")
    G.aggregate_fused(g, K, d, h, dtype, ld, T(left), T(right), True, fused, G.F32, W)
    assert np.abs(host(fused) - fin).max() <= 1e-5
    ldb = G.padded_ld(W, G.BF16)
    fb = torch.full((n, ldb), -1, dtype=torch.int16, device="cuda")
    G.aggregate_fused(g, K, d, h, dtype, ld, T(left), T(right), True, fb, G.BF16, ldb)
    hb = host(fb)
    assert np.all(hb[:, W:] == 0)
    assert np.all(np.abs(G.bf16_to_f32(hb[:, :W]) - fin) <= 2.0 ** -8 * np.abs(fin) + 1e-5)
    # empty rows: zero output, zero max and den (ref_fp32.cpp:11-13)
    empty = np.diff(row.astype(np.int64)) == 0
    if empty.any():
        assert np.all(host(fused)[empty] == 0) and np.all(host(den)[empty] == 0) and np.all(host(mx)[empty] == 0)


@pytest.mark.parametrize("K,d", [(8, 32), (1, 47), (4, 40)])
def test_fixed_p_aggregate(dev, K, d):
    """The reference's fixed-p operator (bench/main.cpp:132): weights and den given."""
    import torch
    row, col = hub_graph(seed=11)
    n = len(row) - 1
    rng = np.random.default_rng(3)
    x = rng.standard_normal((n, 48)).astype(np.float32)
    p = random_layer(rng, 48, K, d)
    o = O.ref_layer(row, col, x, p.w, p.al, p.ar, K, d, False, want_p=True)
    g = G.DeviceGraph(row, col)
    W = K * d
    ld = G.padded_ld(W, G.F32)
    hz = np.zeros((n, ld), np.float32)
    hz[:, :W] = o["z"]
    out = torch.empty((n, W), dtype=torch.float32, device="cuda")
    den = torch.empty((n, K), dtype=torch.float32, device="cuda")
    G.standard_aggregate(g, K, d, T(hz), G.F32, ld, None, None, out, W, den, None,
                         fixed_p=T(o["p"]), fixed_den=T(o["den"]))
    oout, oden = O.standard_aggregate(row, col, o["z"], None, None, None, K, d, fixed_p=o["p"], fixed_den=o["den"])
    assert np.array_equal(host(den), oden)
    assert np.abs(host(out) - oout).max() <= 1e-5 * max(1, np.abs(oout).max())


# ------------------------------------------------------------ layers and model
@pytest.mark.parametrize("D", [17, 33, 128, 256])
def test_boundary_layers_fp32_match_r0(dev, golden, D):
    """The 64 D/K/d cases of baseline/tests/boundaries.cpp, FP32 path vs the reference's R0."""
    import torch
    b = np.load(golden / "boundary.npz")
    row, col, x = O.boundary_graph(D)
    g = G.DeviceGraph(row, col)
    for K in (1, 2, 4, 8):
        for d in (7, 32, 40, 47):
            w, al, ar = O.boundary_params(D, K, d)
            layer = G.DeviceLayer(G.Param(D, K, d, w, al, ar))
            W = K * d
            ld = G.padded_ld(W, G.F32)
            h = torch.empty((35, ld), dtype=torch.float32, device="cuda")
            lr = torch.empty((2, 35, K), dtype=torch.float32, device="cuda")
            out = torch.empty((35, W), dtype=torch.float32, device="cuda")
            G.standard_layer(g, layer, T(x), D, G.PATH_STANDARD_FP32, False, h, lr[0], lr[1], out, G.F32, W)
            e = O.errors(b[f"ref_{D}_{K}_{d}"], host(out))
            assert e["max_abs"] <= 1e-5, (K, d, e)
            assert np.all(host(out)[0] == 0)  # degree-0 row
            # BF16 path: finite, and within the BF16 gate of R0 where it applies
            xb = dev_bf16(x, G.padded_ld(D, G.BF16))
            hb = torch.empty((35, G.padded_ld(W, G.BF16)), dtype=torch.int16, device="cuda")
            ob = torch.empty((35, W), dtype=torch.float32, device="cuda")
            G.standard_layer(g, layer, xb, G.padded_ld(D, G.BF16), G.PATH_STANDARD_BF16, False, hb, lr[0], lr[1],
                             ob, G.F32, W)
            got = host(ob)
            assert np.isfinite(got).all() and np.all(got[0] == 0)
            if f"b0bf16_{D}_{K}_{d}" in b:
                assert rel_l2(b[f"b0bf16_{D}_{K}_{d}"], got) <= 1e-2


def _model(cfg_graph, model_params, path):
    g = G.DeviceGraph(cfg_graph.row, cfg_graph.col)
    layers = [G.DeviceLayer(p) for p in model_params]
    return g, layers, G.DeviceModel(g, layers, path)


def _forward(m, x):
    import torch
    n = x.shape[0]
    logits = torch.empty((n, m.classes), dtype=torch.float32, device="cuda")
    m.forward(T(x), logits, False, False)
    return host(logits)


def _smoke_inputs(golden):
    import tempfile
    from pathlib import Path
    from golden.make_golden import write_smoke1024
    with tempfile.TemporaryDirectory() as d:
        p = Path(d) / "s.gatbin"
        write_smoke1024(p)
        return G.load_graph(p)


@pytest.mark.parametrize("name", ["config1", "smoke1024_seed11"])
def test_model_matches_reference_goldens(dev, golden, name):
    import configs
    ref = np.load(golden / f"{name}.npz")
    if name == "config1":
        cfg = configs.make("c1")
        graph, params = cfg.graph, cfg.model
    else:
        graph, params = _smoke_inputs(golden), G.random_model(128, 40, 11)
    # FP32 path: north-star gate max-abs <= 1e-5 against R0
    _, _, m32 = _model(graph, params, G.PATH_STANDARD_FP32)
    got32 = _forward(m32, graph.x)
    e = O.errors(ref["ref_logits"], got32)
    assert e["max_abs"] <= 1e-5, e
    # BF16 path: rel-L2 <= 1e-2 against R0, and close to the reference's own B0 BF16
    _, _, m16 = _model(graph, params, G.PATH_STANDARD_BF16)
    got16 = _forward(m16, graph.x)
    assert rel_l2(ref["ref_logits"], got16) <= 1e-2
    assert rel_l2(ref["b0bf16_logits"], got16) <= 1e-2
    # and to the B0 restatement that also rounds H to BF16 as the device does
    inp = graph.x
    for l, p in enumerate(params):
        inp = O.b0_layer(graph.row, graph.col, inp, p.w, p.al, p.ar, p.heads, p.dim, l < 2, bf16=True,
                         round_z=True)["out"]
    assert rel_l2(inp, got16) <= 3e-3


def test_model_host_buffers_e2e(dev):
    """model_forward with host input/output (the reference-facing call)."""
    import torch
    import configs
    cfg = configs.make("c1")
    _, _, m = _model(cfg.graph, cfg.model, G.PATH_STANDARD_BF16)
    xh = torch.from_numpy(cfg.graph.x).pin_memory()
    lh = torch.empty((cfg.graph.n, m.classes), dtype=torch.float32).pin_memory()
    m.forward(xh, lh, True, True)
    dev_logits = _forward(m, cfg.graph.x)
    assert np.array_equal(lh.numpy(), dev_logits)


def test_model_forward_async_pipeline(dev):
    """Pipelined host-to-host forwards (two slots, own copy streams): every
    request's logits equal the synchronous forward's, bit for bit."""
    import torch
    import configs
    cfg = configs.make("c1")
    _, _, m = _model(cfg.graph, cfg.model, G.PATH_STANDARD_BF16)
    xs = [torch.from_numpy((cfg.graph.x * s).astype(np.float32)).pin_memory() for s in (1.0, -0.5, 2.0)]
    outs = [torch.empty((cfg.graph.n, m.classes), dtype=torch.float32).pin_memory() for _ in xs]
    st = torch.cuda.current_stream()
    for x, o in zip(xs, outs):
        m.forward_async(x, o, st)
    m.join(st)
    torch.cuda.synchronize()
    G.check_device()
    for x, o in zip(xs, outs):
        want = _forward(m, x.numpy())
        assert np.array_equal(o.numpy(), want)


@pytest.mark.slow
def test_config2_model(dev):
    """arxiv-shaped power-law graph (hub rows split into segments)."""
    import configs
    cfg = configs.make("c2")
    g, _, m16 = _model(cfg.graph, cfg.model, G.PATH_STANDARD_BF16)
    assert g.info()["n_hub"] > 0
    got16 = _forward(m16, cfg.graph.x)
    model = [(p.w, p.al, p.ar, p.heads, p.dim) for p in cfg.model]
    ref = O.ref_chain(cfg.graph.row, cfg.graph.col, cfg.graph.x, model)[2]["out"]
    assert rel_l2(ref, got16) <= 1e-2
    _, _, m32 = _model(cfg.graph, cfg.model, G.PATH_STANDARD_FP32)
    got32 = _forward(m32, cfg.graph.x)
    e = O.errors(ref, got32)
    assert e["max_abs"] <= 1e-5, e


@pytest.mark.parametrize("n,width,ld_in", [(1000, 100, 100), (333, 47, 48), (257, 13, 13), (64, 256, 260)])
def test_convert_bit_exact(dev, n, width, ld_in):
    """gat_b200_convert (16-byte path when rows allow it, else the pairwise one) equals the
    host RNE bit for bit, padding columns zero; ties, subnormals, infinities and NaN included."""
    import torch
    rng = np.random.default_rng(n + width)
    x = rng.standard_normal((n, ld_in)).astype(np.float32)
    specials = np.array([np.inf, -np.inf, np.nan, 1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8, -0.0, 1e-40, 3.4e38],
                        np.float32)
    x.reshape(-1)[: len(specials)] = specials
    ld_out = G.padded_ld(width, G.BF16)
    out = torch.full((n, ld_out), -1, dtype=torch.int16, device="cuda")
    G.convert(n, width, T(x), ld_in, out, ld_out)
    got = host(out)
    want = G.rne(np.ascontiguousarray(x[:, :width]))
    assert np.array_equal(got[:, :width], want)
    assert not got[:, width:].any()


@pytest.mark.parametrize("scenario", range(5))
@pytest.mark.parametrize("dtype", [G.F32, G.BF16])
def test_adversarial_scores(dev, scenario, dtype):
    """The reference's adversarial score cases (baseline/tests/boundaries.cpp:45-51) on its
    17-feature boundary graph with 8 heads of 32: equal scores, a late +1000 peak after -1000
    sources, increasing scores, and common offsets of +10000 / -10000. Outputs finite, the
    max bit-exact, den >= 1 on non-empty rows and 0 on empty ones, and the online-softmax
    kernels equal to the oracle."""
    import torch
    row, col, _ = O.boundary_graph(17)
    n, K, d = len(row) - 1, 8, 32
    W = K * d
    i = np.arange(n, dtype=np.float32)[:, None]
    h = np.arange(K, dtype=np.float32)[None, :]
    left = np.broadcast_to({3: np.float32(10000), 4: np.float32(-10000)}.get(scenario, h - 4), (n, K))
    right = [np.zeros((n, K)), np.where(i == n - 1, 1000.0, -1000.0) + 0 * h, (i - 17) + 0 * h,
             np.sin(i + h) * 8, np.sin(i + h) * 8][scenario]
    left = np.ascontiguousarray(left, np.float32)
    right = np.ascontiguousarray(right, np.float32)
    z = ((np.arange(n * W) % 9) * np.float32(0.1)).astype(np.float32).reshape(n, W)
    ld = G.padded_ld(W, dtype)
    if dtype == G.BF16:
        z = O.quantize(z)
        hz = dev_bf16(z, ld)
    else:
        hz = T(z)
    g = G.DeviceGraph(row, col)
    out = torch.empty((n, W), dtype=torch.float32, device="cuda")
    den = torch.empty((n, K), dtype=torch.float32, device="cuda")
    mx = torch.empty((n, K), dtype=torch.float32, device="cuda")
    G.standard_aggregate(g, K, d, hz, dtype, ld, T(left), T(right), out, W, den, mx)
    omax = O.max_prescan(row, col, left, right, K)
    oout, oden = O.standard_aggregate(row, col, z, left, right, omax, K, d)
    got_out, got_den = host(out), host(den)
    assert np.all(np.isfinite(got_out)) and np.all(np.isfinite(got_den))
    assert np.array_equal(host(mx), omax)
    empty = np.diff(row.astype(np.int64)) == 0
    assert np.all(got_den[empty] == 0) and np.all(got_den[~empty] >= 1)
    assert np.abs(got_den - oden).max() <= 1e-5 * max(1, np.abs(oden).max())
    assert np.abs(got_out - oout).max() <= 1e-5 * max(1, np.abs(oout).max())
    fused = torch.empty((n, W), dtype=torch.float32, device="cuda")
    G.aggregate_fused(g, K, d, hz, dtype, ld, T(left), T(right), False, fused, G.F32, W)
    fin = O.finish(oout, oden, K, d, False)
    assert np.all(np.isfinite(host(fused)))
    assert np.abs(host(fused) - fin).max() <= 1e-5 * max(1, np.abs(fin).max())
    g.close()
