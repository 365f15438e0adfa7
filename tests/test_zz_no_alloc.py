"""The aggregation entry point that allocates no device memory.

gat_b200_aggregate_fused_noalloc serves callers that cannot allocate device
memory themselves (a plugin running inside another framework whose allocator
owns the GPU, or a serving loop where cudaMalloc would synchronize the device).
It must give the same result as gat_b200_aggregate_fused, the regular entry
point, on graphs whose long rows cross its internal edge ranges, and keep doing
so when called twice in a row (its scratch array keeps the previous call's
contents). This file is collected last so that a failure here leaves every
other test already run; it also passes when run on its own.
"""
import numpy as np
import pytest

import gatb200 as G

pytestmark = pytest.mark.gpu


def _graph(kind):
    rng = np.random.default_rng(17)
    if kind == "hubs":
        n, hubs = 3000, (2900, 2500, 1800, 700)
        row, col = [0], []
        for i in range(n):
            deg = hubs[i % len(hubs)] if i % 500 == 7 else int(rng.integers(0, 6))
            col.extend(sorted(rng.choice(n, size=deg, replace=False).tolist()))
            row.append(len(col))
        return np.array(row, np.uint64), np.array(col, np.uint32)
    if kind == "powerlaw":
        return G.synth_powerlaw_graph(20000, 400000, 9000, 2.1, 5)
    if kind == "large":
        # more than 7936 * 1024 edges: the range count is capped and every
        # range grows beyond 1024 edges, as on the benchmark graphs
        return G.synth_powerlaw_graph(300_000, 9_000_000, 20_000, 2.1, 7)
    return G.synth_uniform_graph(1024, 15, 1)


@pytest.mark.parametrize("kind,K,d,out_dtype,h_dtype", [
    (kind, K, d, o, G.BF16) for kind in ("hubs", "powerlaw", "uniform")
    for K, d, o in ((8, 32, G.BF16), (1, 47, G.F32), (4, 40, G.BF16))
] + [("hubs", 8, 32, G.F32, G.F32), ("powerlaw", 1, 47, G.F32, G.F32), ("large", 8, 32, G.BF16, G.BF16),
     ("large", 1, 47, G.F32, G.BF16)])
def test_noalloc_matches_regular_entry_point(dev, kind, K, d, out_dtype, h_dtype):
    import torch
    row, col = _graph(kind)
    n, e, W = len(row) - 1, len(col), K * d
    rng = np.random.default_rng(K * 1000 + d)
    ldh = G.padded_ld(W, h_dtype)
    hf = rng.standard_normal((n, W)).astype(np.float32)
    if h_dtype == G.BF16:
        hz = np.zeros((n, ldh), np.uint16)
        hz[:, :W] = G.rne(hf)
        h = torch.from_numpy(hz.view(np.int16)).cuda()
    else:
        hz = np.zeros((n, ldh), np.float32)
        hz[:, :W] = hf
        h = torch.from_numpy(hz).cuda()
    left = torch.from_numpy(rng.standard_normal((n, K)).astype(np.float32)).cuda()
    right = torch.from_numpy(rng.standard_normal((n, K)).astype(np.float32)).cuda()
    ldo = G.padded_ld(W, out_dtype)
    odt = torch.int16 if out_dtype == G.BF16 else torch.float32

    g = G.DeviceGraph(row, col)
    ref = torch.zeros((n, ldo), dtype=odt, device="cuda")
    G.aggregate_fused(g, K, d, h, h_dtype, ldh, left, right, True, ref, out_dtype, ldo)

    row_d = torch.from_numpy(row.view(np.int64)).cuda()
    col_d = torch.from_numpy(col.view(np.int32)).cuda()
    for call in range(2):  # the second call reuses the scratch left by the first
        out = torch.full((n, ldo), 3, dtype=odt, device="cuda")
        G.aggregate_fused_noalloc(n, e, row_d, col_d, K, d, h, h_dtype, ldh, left, right, True, out, out_dtype, ldo)
        torch.cuda.synchronize()
        G.check_device()
        a, b = ref.cpu().numpy(), out.cpu().numpy()
        if out_dtype == G.BF16:
            a = G.bf16_to_f32(a.view(np.uint16))
            b = G.bf16_to_f32(b.view(np.uint16))
            # same math, different summation order: at most one BF16 rounding apart
            tol = 2.0 ** -7 * np.abs(a) + 1e-5
        else:
            tol = 1e-5 * np.maximum(1.0, np.abs(a))
        assert np.all(np.abs(a - b) <= tol), (call, float(np.abs(a - b).max()))


@pytest.mark.parametrize("kind,K,d", [("hubs", 8, 32), ("powerlaw", 1, 47), ("uniform", 4, 40)])
def test_noalloc_matches_oracle(dev, kind, K, d):
    """The same entry point against the CPU oracle's max prescan, standard
    aggregate and finish (the reference's B0 stages) on the same inputs:
    FP32 output within 1e-5 relative to the largest value (the same math,
    another summation order)."""
    import torch
    import oracle as O
    row, col = _graph(kind)
    n, e, W = len(row) - 1, len(col), K * d
    rng = np.random.default_rng(K * 100 + d)
    ldh = G.padded_ld(W, G.BF16)
    hb = G.rne(rng.standard_normal((n, W)).astype(np.float32))
    hz = np.zeros((n, ldh), np.uint16)
    hz[:, :W] = hb
    L = rng.standard_normal((n, K)).astype(np.float32)
    R = rng.standard_normal((n, K)).astype(np.float32)
    z = G.bf16_to_f32(hb)
    mx = O.max_prescan(row, col, L, R, K)
    agg, den = O.standard_aggregate(row, col, z, L, R, mx, K, d)
    want = O.finish(agg, den, K, d, True)
    out = torch.zeros((n, W), dtype=torch.float32, device="cuda")
    G.aggregate_fused_noalloc(n, e, torch.from_numpy(row.view(np.int64)).cuda(),
                              torch.from_numpy(col.view(np.int32)).cuda(), K, d,
                              torch.from_numpy(hz.view(np.int16)).cuda(), G.BF16, ldh, torch.from_numpy(L).cuda(),
                              torch.from_numpy(R).cuda(), True, out, G.F32, W)
    torch.cuda.synchronize()
    G.check_device()
    got = out.cpu().numpy()
    assert np.abs(got - want).max() <= 1e-5 * max(1.0, float(np.abs(want).max())), float(np.abs(got - want).max())


def test_noalloc_rejects_bad_arguments(dev):
    import torch
    row, col = _graph("uniform")
    n, e = len(row) - 1, len(col)
    row_d = torch.from_numpy(row.view(np.int64)).cuda()
    col_d = torch.from_numpy(col.view(np.int32)).cuda()
    h = torch.zeros((n, 256), dtype=torch.int16, device="cuda")
    lr = torch.zeros((n, 8), dtype=torch.float32, device="cuda")
    out = torch.zeros((n, 256), dtype=torch.int16, device="cuda")
    with pytest.raises(G.GatError, match="heads <=8"):
        G.aggregate_fused_noalloc(n, e, row_d, col_d, 9, 32, h, G.BF16, 256, lr, lr, True, out, G.BF16, 256)
    with pytest.raises(G.GatError, match="bad output dtype"):
        G.aggregate_fused_noalloc(n, e, row_d, col_d, 8, 32, h, G.BF16, 256, lr, lr, True, out, 7, 256)
    with pytest.raises(G.GatError, match="exceed the maximum"):
        G.aggregate_fused_noalloc(n, 600_000_000, row_d, col_d, 8, 32, h, G.BF16, 256, lr, lr, True, out, G.BF16,
                                  256)
