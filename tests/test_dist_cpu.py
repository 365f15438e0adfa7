"""Host logic of the row-partitioned multi-GPU forward, on CPU with gloo.

Each of two ranks builds its slice exactly as the GPU path does
(dist.partition / slice_local / configs.make_part), runs the three layers with
the CPU oracle on its own rows, exchanges the projected features and R with a
gloo all-gather into the padded table, and the gathered logits must equal the
single-process oracle bit for bit: every row sees the same sources in the same
order, so the arithmetic is identical.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as tdist
import torch.multiprocessing as mp

import configs
import dist as gdist
import gatb200 as G
import oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, name, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        part = configs.make_part(name, rank, world)
        row_loc, col_loc, n_max = gdist.slice_local(part.row, part.col_rows, part.cuts, rank)
        n_loc = len(row_loc) - 1
        x = part.x_rows
        for l, p in enumerate(part.model):
            K, d, W = p.heads, p.dim, p.width
            o = O.ref_layer(np.zeros(n_loc + 1, np.uint64), np.zeros(0, np.uint32), x, p.w, p.al, p.ar, K, d, False)
            z_pad = np.zeros((n_max, W), np.float32)
            r_pad = np.zeros((n_max, K), np.float32)
            z_pad[:n_loc] = o["z"]
            r_pad[:n_loc] = o["right"]
            zs = [torch.zeros((n_max, W)) for _ in range(world)]
            rs = [torch.zeros((n_max, K)) for _ in range(world)]
            tdist.all_gather(zs, torch.from_numpy(z_pad))
            tdist.all_gather(rs, torch.from_numpy(r_pad))
            z_full = torch.cat(zs).numpy()
            r_full = torch.cat(rs).numpy()
            mx = O.max_prescan(row_loc, col_loc, o["left"], r_full, K)
            out, den = O.standard_aggregate(row_loc, col_loc, z_full, o["left"], r_full, mx, K, d)
            x = O.finish(out, den, K, d, l < 2)
        pad = np.zeros((n_max, x.shape[1]), np.float32)
        pad[:n_loc] = x
        outs = [torch.zeros_like(torch.from_numpy(pad)) for _ in range(world)]
        tdist.all_gather(outs, torch.from_numpy(pad))
        if rank == 0:
            full = np.concatenate([outs[k].numpy()[: int(part.cuts[k + 1] - part.cuts[k])] for k in range(world)])
            q.put(full)
    finally:
        tdist.destroy_process_group()


def _single_process_reference(name):
    cfg = configs.make(name)
    x = cfg.graph.x
    for l, p in enumerate(cfg.model):
        o = O.ref_layer(cfg.graph.row, cfg.graph.col, x, p.w, p.al, p.ar, p.heads, p.dim, False)
        mx = O.max_prescan(cfg.graph.row, cfg.graph.col, o["left"], o["right"], p.heads)
        out, den = O.standard_aggregate(cfg.graph.row, cfg.graph.col, o["z"], o["left"], o["right"], mx, p.heads,
                                        p.dim)
        x = O.finish(out, den, p.heads, p.dim, l < 2)
    return x


def test_partition_balances_edges():
    g = configs.make_graph("c2", features=False)
    for world in (2, 4, 8):
        cuts = gdist.partition(g.row, world)
        assert cuts[0] == 0 and cuts[-1] == g.n and np.all(np.diff(cuts) > 0)
        edges = np.diff(g.row[cuts].astype(np.int64))
        assert edges.max() <= g.e / world + 13162  # at most one row over the even share


def test_slice_remaps_sources_into_padded_table():
    g = configs.make_graph("c2", features=False)
    world = 4
    cuts = gdist.partition(g.row, world)
    n_max = int(np.diff(cuts).max())
    for rank in range(world):
        row_loc, col_loc, nm = gdist.slice_graph(g.row, g.col, cuts, rank)
        assert nm == n_max
        lo, hi = cuts[rank], cuts[rank + 1]
        src = g.col[int(g.row[lo]):int(g.row[hi])].astype(np.int64)
        owner = col_loc.astype(np.int64) // n_max
        back = cuts[owner] + col_loc.astype(np.int64) % n_max
        assert np.array_equal(back, src)
        assert np.all(col_loc.astype(np.int64) % n_max < np.diff(cuts)[owner])


def test_make_part_matches_whole_graph():
    g = configs.make_graph("c2")
    for rank in range(3):
        p = configs.make_part("c2", rank, 3)
        assert np.array_equal(p.row, g.row)
        assert np.array_equal(p.col_rows, g.col[int(g.row[p.lo]):int(g.row[p.hi])])
        assert np.array_equal(p.x_rows, g.x[p.lo:p.hi])


@pytest.mark.slow
def test_two_rank_forward_equals_single_process():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, "c2", q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    want = _single_process_reference("c2")
    assert np.array_equal(got, want)
