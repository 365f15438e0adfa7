"""RMAT stress configuration (c5): generator and sampled FP64 parity.

* gat_b200_synth_rmat (GPU) equals a numpy restatement of the same
  counter-based draws, quadrant rule, self loops and de-duplication, bit for
  bit, on small graphs.
* A full R0 oracle of c5 (2^24 nodes, ~0.5 G edges) does not fit the host, so
  each layer is checked on sampled rows with their complete neighbourhoods:
  the layer's BF16 input rows of every neighbour are read back from the GPU,
  the layer is recomputed in FP64 (BF16 W, FP64 scores, softmax and sums) and
  compared with the GPU's output rows. Sampled rows: random ones plus rows at
  degree quantiles, the largest hub included. Gate: relative L2 over all
  sampled rows <= 1e-2 (the BF16 gate against R0), <= 3e-2 for every row.
"""
import numpy as np
import pytest

import configs
import gatb200 as G

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


def _bf16_rows(t, idx, width):
    """BF16 rows idx of device tensor t (int16 storage) as float64."""
    import torch
    sel = t.index_select(0, torch.from_numpy(np.asarray(idx, np.int64)).cuda()).cpu().numpy()
    return G.bf16_to_f32(sel.view(np.uint16)[:, :width]).astype(np.float64)


def _layer_fp64(xn, xi, w, al, ar, heads, dim, hidden):
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


def _sampled_check(name, nsample=48, seed=17):
    import torch
    cfg = configs.make(name)
    gr = cfg.graph
    n = gr.n
    deg = np.diff(gr.row.astype(np.int64))
    rng = np.random.default_rng(seed)
    order = np.argsort(deg, kind="stable")
    quant = [order[int(q * (n - 1))] for q in (0.5, 0.9, 0.99, 0.999, 0.9999)] + [int(order[-1])]
    rows = np.unique(np.concatenate([rng.choice(n, nsample, replace=False), quant]))

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
    errs, refs = [], []
    for l, p in enumerate(cfg.model):
        hidden = l < 2
        xin, ldin = xs_[l], (ld0 if l == 0 else ldx)
        out = xs_[l + 1] if hidden else logits
        G.standard_layer(g, layers[l], xin, ldin, G.PATH_STANDARD_BF16, hidden, h, left, right, out,
                         G.BF16 if hidden else G.F32, ldx if hidden else p.width)
        torch.cuda.synchronize()
        G.check_device()
        w = G.bf16_to_f32(G.rne(p.w)).astype(np.float64)
        al, ar = p.al.astype(np.float64), p.ar.astype(np.float64)
        if hidden:
            got = _bf16_rows(out, rows, p.width)
        else:
            got = logits.index_select(0, torch.from_numpy(rows.astype(np.int64)).cuda()).cpu().numpy().astype(
                np.float64)
        for k, i in enumerate(rows):
            nb = gr.col[int(gr.row[i]):int(gr.row[i + 1])]
            xn = _bf16_rows(xin, nb, p.in_)
            xi = _bf16_rows(xin, [i], p.in_)[0]
            ref = _layer_fp64(xn, xi, w, al, ar, p.heads, p.dim, hidden)
            errs.append(got[k] - ref)
            refs.append(ref)
            rel = np.linalg.norm(got[k] - ref) / max(np.linalg.norm(ref), 1e-30)
            assert rel <= 3e-2, (name, l, int(i), int(deg[i]), rel)
    e = np.concatenate(errs)
    r = np.concatenate(refs)
    rel_all = np.linalg.norm(e) / np.linalg.norm(r)
    for lay in layers:
        lay.close()
    g.close()
    return rel_all, int(deg.max()), len(rows)


@pytest.mark.parametrize("name", ["c5s", "c5"])
def test_rmat_sampled_rows_fp64(dev, name):
    rel, max_deg, k = _sampled_check(name)
    assert rel <= 1e-2, (name, rel, max_deg, k)
