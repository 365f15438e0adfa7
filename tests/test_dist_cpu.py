"""Host logic of the row-partitioned multi-GPU forward, on CPU with gloo.

Each of two ranks builds its slice exactly as the GPU path does
(dist.Layout / slice_chunk / configs.make_part), runs the three layers with
the CPU oracle on its own rows, exchanges the projected features and R with a
gloo all-gather into the padded table, and the gathered logits must equal the
single-process oracle bit for bit: every row sees the same sources in the same
order, so the arithmetic is identical.
"""
import functools
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


def _rank_main(rank, world, port, name, q, chunks=4):
    """Rank `rank` of the pipelined partitioned forward, with the oracle as the
    arithmetic: chunk-major feature table, one all-gather per chunk."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tdist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        part = configs.make_part(name, rank, world)
        lay = gdist.Layout(part.row, world, chunks, part.cuts)
        cm = lay.chunk_max
        slices = [lay.slice_chunk(part.row, part.col_rows, rank, c) for c in range(chunks)]
        bounds = [lay.chunk_rows(rank, c) for c in range(chunks)]
        n_loc = part.hi - part.lo
        x = part.x_rows
        for l, p in enumerate(part.model):
            K, d, W = p.heads, p.dim, p.width
            o = O.ref_layer(np.zeros(n_loc + 1, np.uint64), np.zeros(0, np.uint32), x, p.w, p.al, p.ar, K, d, False)
            z_tab = np.zeros((lay.n_table, W), np.float32)
            r_tab = np.zeros((lay.n_table, K), np.float32)
            for c, (a_, b_) in enumerate(bounds):
                zb = np.zeros((cm, W), np.float32)
                rb = np.zeros((cm, K), np.float32)
                zb[: b_ - a_] = o["z"][a_:b_]
                rb[: b_ - a_] = o["right"][a_:b_]
                zs = [torch.zeros((cm, W)) for _ in range(world)]
                rs = [torch.zeros((cm, K)) for _ in range(world)]
                tdist.all_gather(zs, torch.from_numpy(zb))
                tdist.all_gather(rs, torch.from_numpy(rb))
                z_tab[c * world * cm:(c + 1) * world * cm] = torch.cat(zs).numpy()
                r_tab[c * world * cm:(c + 1) * world * cm] = torch.cat(rs).numpy()
            nxt = np.zeros((n_loc, W), np.float32)
            for c, (a_, b_) in enumerate(bounds):
                if b_ == a_:
                    continue
                rl, cl = slices[c]
                left = o["left"][a_:b_]
                mx = O.max_prescan(rl, cl, left, r_tab, K)
                out, den = O.standard_aggregate(rl, cl, z_tab, left, r_tab, mx, K, d)
                nxt[a_:b_] = O.finish(out, den, K, d, l < 2)
            x = nxt
        n_max = int(np.diff(part.cuts).max())
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


def test_layout_slots_round_trip():
    """Every source's table row maps back to it; chunk slices cover every edge once."""
    g = configs.make_graph("c2", features=False)
    for world in (2, 4, 8):
        for chunks in (1, 4):
            lay = gdist.Layout(g.row, world, chunks)
            src = np.arange(g.n)
            slots = lay.slots(src).astype(np.int64)
            assert len(np.unique(slots)) == g.n and slots.max() < lay.n_table
            blk, i = slots // lay.chunk_max, slots % lay.chunk_max
            c, r = blk // world, blk % world
            assert np.array_equal(lay.ccuts[r, c] + i, src)
            assert np.all(lay.ccuts[r, c] + i < lay.ccuts[r, c + 1])
            for rank in range(world):
                lo, hi = int(lay.cuts[rank]), int(lay.cuts[rank + 1])
                col_rows = g.col[int(g.row[lo]):int(g.row[hi])]
                got = []
                for ch in range(chunks):
                    rl, cl = lay.slice_chunk(g.row, col_rows, rank, ch)
                    a, b = lay.chunk_rows(rank, ch)
                    assert len(rl) == b - a + 1 and int(rl[-1]) == len(cl)
                    got.append(cl)
                assert np.array_equal(np.concatenate(got), lay.slots(col_rows))


def test_make_part_matches_whole_graph():
    g = configs.make_graph("c2")
    for rank in range(3):
        p = configs.make_part("c2", rank, 3)
        assert np.array_equal(p.row, g.row)
        assert np.array_equal(p.col_rows, g.col[int(g.row[p.lo]):int(g.row[p.hi])])
        assert np.array_equal(p.x_rows, g.x[p.lo:p.hi])


@functools.lru_cache(maxsize=None)
def _reference_c2():
    return _single_process_reference("c2")


@pytest.mark.slow
@pytest.mark.parametrize("world,chunks", [(2, 4), (8, 2)])
def test_partitioned_forward_equals_single_process(world, chunks):
    """The rank-local pipeline at the bench's smallest and largest world sizes:
    the gathered logits equal the single-process oracle bit for bit."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, "c2", q, chunks)) for r in range(world)]
    for p in procs:
        p.start()
    got = q.get(timeout=600)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert np.array_equal(got, _reference_c2())


def test_multi_gpu_c_abi_host_checks(tmp_path):
    """Host-side checks of the communicator and the partitioned model (no GPU
    touched): bad world sizes and ranks are refused, and a rank whose rank 0
    never publishes the communicator id gives up after its timeout with
    GAT_B200_ETIMEOUT instead of waiting for ever."""
    import ctypes as C
    import time
    h = C.c_void_p()
    rc = G._lib.gat_b200_comm_create(None, 9, 0, C.byref(h))
    assert rc == G.EINVAL and b"world size" in G._lib.gat_b200_last_error()
    rc = G._lib.gat_b200_comm_create(None, 2, 2, C.byref(h))
    assert rc == G.EINVAL and b"rank outside" in G._lib.gat_b200_last_error()
    t0 = time.time()
    with pytest.raises(G.GatError, match="no unique id") as ei:
        G.Comm(2, 1, path=str(tmp_path / "never_written"), timeout_ms=300)
    assert ei.value.code == G.ETIMEOUT and time.time() - t0 < 10
    rc = G._lib.gat_b200_part_model_create(None, 0, None, None, None, 0, 1, None, C.byref(h))
    assert rc == G.EINVAL
    # the model's switches refuse a null handle with a message
    for fn, arg, what in ((G._lib.gat_b200_part_model_set_layer2_exchange, 1, b"set_layer2_exchange"),
                          (G._lib.gat_b200_part_model_set_overlap, 0, b"set_overlap"),
                          (G._lib.gat_b200_part_model_enable_timing, 1, b"enable_timing")):
        assert fn(None, arg) == G.EINVAL and what in G._lib.gat_b200_last_error()


def _rank_fails(rank, world, port, q):
    """Rank 1 dies before the layer exchange (it raises after joining); rank 0
    must learn of it from the process group's deadline, not hang."""
    import datetime
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    tdist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        raise RuntimeError("injected rank failure before the exchange")
    t0 = time.time()
    try:
        zs = [torch.zeros(4) for _ in range(world)]
        tdist.all_gather(zs, torch.ones(4))
        q.put(("no error", time.time() - t0))
    except Exception as e:  # the exchange of a dead peer fails within the deadline
        q.put((type(e).__name__, time.time() - t0))


def test_failed_rank_is_detected_by_the_exchange_deadline():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_fails, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    kind, waited = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert kind != "no error" and waited < 60, (kind, waited)
    assert procs[1].exitcode != 0 and procs[0].exitcode == 0
