"""Sampled complete-neighbourhood FP64 check of a three-layer forward.

A full R0 oracle of the large configurations (c4: 126M edges, c5: 0.5G
edges) is too slow or too large for the host, so each layer is checked on
sampled destination rows with their complete neighbourhoods: the layer's BF16
input rows of every neighbour are read back from the GPU, the layer is
recomputed in FP64 (BF16 W, FP64 scores, softmax and sums) and compared with
the GPU's output rows. Sampled rows: random ones plus the rows at the
50/90/99/99.9/99.99 % degree quantiles and the largest hub. The per-layer
semantics are R0's (baseline/src/ref_fp32.cpp:3-26) with the BF16 roundings of
B0 (baseline/src/baseline_standard.cpp:3-6, common.cpp:85-93).

This module is test infrastructure (imported by the gpu tests only).
"""
import numpy as np

import gatb200 as G


def sample_rows(row, nsample=48, seed=17):
    """Random rows plus the degree quantiles and the largest hub (sorted, unique)."""
    deg = np.diff(row.astype(np.int64))
    n = len(deg)
    rng = np.random.default_rng(seed)
    order = np.argsort(deg, kind="stable")
    quant = [order[int(q * (n - 1))] for q in (0.5, 0.9, 0.99, 0.999, 0.9999)] + [int(order[-1])]
    return np.unique(np.concatenate([rng.choice(n, nsample, replace=False), quant]))


def bf16_rows(t, idx, width):
    """BF16 rows idx of device tensor t (int16 storage) as float64."""
    import torch
    sel = t.index_select(0, torch.from_numpy(np.asarray(idx, np.int64)).to(t.device)).cpu().numpy()
    return G.bf16_to_f32(sel.view(np.uint16)[:, :width]).astype(np.float64)


def layer_fp64(xn, xi, w, al, ar, heads, dim, hidden):
    """FP64 GAT layer for one destination row: xn = neighbour input rows, xi = its own."""
    z = xn @ w
    zi = xi @ w
    zh = z.reshape(len(xn), heads, dim)
    L = (zi.reshape(heads, dim) * al.reshape(heads, dim)).sum(1)
    R = (zh * ar.reshape(1, heads, dim)).sum(2)
    s = L[None, :] + R
    s = np.where(s > 0, s, 0.2 * s)
    p = np.exp(s - s.max(0, keepdims=True))
    alpha = p / p.sum(0, keepdims=True)
    out = (alpha[:, :, None] * zh).sum(0).reshape(-1)
    return np.where(out < 0, np.expm1(out), out) if hidden else out


def check_layer(row, col, rows, xin, out_rows, p, hidden):
    """FP64 recomputation of one layer on `rows` against the GPU's out_rows
    (float64 [len(rows), width]). xin: the layer's BF16 input on the device.
    Returns (errors, references, per-row relative L2)."""
    w = G.bf16_to_f32(G.rne(p.w)).astype(np.float64)
    al, ar = p.al.astype(np.float64), p.ar.astype(np.float64)
    errs, refs, rels = [], [], []
    for k, i in enumerate(rows):
        nb = col[int(row[i]):int(row[i + 1])]
        xn = bf16_rows(xin, nb, p.in_)
        xi = bf16_rows(xin, [i], p.in_)[0]
        ref = layer_fp64(xn, xi, w, al, ar, p.heads, p.dim, hidden)
        errs.append(out_rows[k] - ref)
        refs.append(ref)
        rels.append(float(np.linalg.norm(out_rows[k] - ref) / max(np.linalg.norm(ref), 1e-30)))
    return errs, refs, rels


def sampled_forward_check(cfg, nsample=48, seed=17):
    """Runs the BF16 three-layer forward of cfg layer by layer through
    gat_b200_standard_layer and checks every layer on sampled rows.
    Returns a dict: rel_l2 over all sampled rows and layers, the worst row
    (layer, row, degree, rel), the number of rows, the largest degree."""
    import torch
    gr = cfg.graph
    n = gr.n
    deg = np.diff(gr.row.astype(np.int64))
    rows = sample_rows(gr.row, nsample, seed)
    g = G.DeviceGraph(gr.row, gr.col)
    layers = [G.DeviceLayer(p) for p in cfg.model]
    ld0 = G.padded_ld(gr.din, G.BF16)
    x0 = torch.zeros((n, ld0), dtype=torch.int16, device="cuda")
    chunk = 1 << 20
    for a in range(0, n, chunk):  # FP32 -> BF16 in slices (bounded device memory)
        b = min(n, a + chunk)
        xs = torch.from_numpy(gr.x[a:b]).cuda()
        G.convert(b - a, gr.din, xs, gr.din, x0[a:b], ld0)
        del xs
    widths = [p.width for p in cfg.model]
    ldh = G.padded_ld(max(widths), G.BF16)
    h = torch.zeros((n, ldh), dtype=torch.int16, device="cuda")
    left = torch.zeros((n, 8), dtype=torch.float32, device="cuda")
    right = torch.zeros((n, 8), dtype=torch.float32, device="cuda")
    ldx = G.padded_ld(max(widths[:2]), G.BF16)
    xs_ = [x0] + [torch.zeros((n, ldx), dtype=torch.int16, device="cuda") for _ in range(2)]
    logits = torch.zeros((n, cfg.model[2].width), dtype=torch.float32, device="cuda")
    errs, refs, worst = [], [], (0, 0, 0, 0.0)
    try:
        for l, p in enumerate(cfg.model):
            hidden = l < 2
            xin, ldin = xs_[l], (ld0 if l == 0 else ldx)
            out = xs_[l + 1] if hidden else logits
            G.standard_layer(g, layers[l], xin, ldin, G.PATH_STANDARD_BF16, hidden, h, left, right, out,
                             G.BF16 if hidden else G.F32, ldx if hidden else p.width)
            torch.cuda.synchronize()
            G.check_device()
            if hidden:
                got = bf16_rows(out, rows, p.width)
            else:
                got = logits.index_select(0, torch.from_numpy(rows.astype(np.int64)).cuda()).cpu().numpy().astype(
                    np.float64)
            e_, r_, rel = check_layer(gr.row, gr.col, rows, xin, got, p, hidden)
            errs += e_
            refs += r_
            k = int(np.argmax(rel))
            if rel[k] > worst[3]:
                worst = (l + 1, int(rows[k]), int(deg[rows[k]]), rel[k])
    finally:
        for lay in layers:
            lay.close()
        g.close()
    e = np.concatenate(errs)
    r = np.concatenate(refs)
    return {"rel_l2": float(np.linalg.norm(e) / np.linalg.norm(r)), "worst": worst, "rows": len(rows),
            "max_degree": int(deg.max())}
