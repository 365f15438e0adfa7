"""Row-partitioned forward on 2 GPUs against the 1-GPU model, with the
exchange done by the projection kernel's peer stores (p2p), by copy-engine
pushes (dma; one and three row chunks each) and by NCCL all-gathers (four
chunks).

Skipped when fewer than two GPUs are visible. Ranks run as child processes
with NCCL's NVLink SHARP (NVLS) disabled and a short process-group timeout.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, name, q, exchange, chunks):
    import datetime
    import torch
    import torch.distributed as tdist
    import configs
    import dist as gdist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    tdist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                             device_id=torch.device("cuda", rank))
    try:
        part = configs.make_part(name, rank, world)
        pm = gdist.PartitionedModel(part.row, part.col_rows, part.model, rank, world,
                                    torch.cuda.current_stream(), tdist, part.cuts, chunks=chunks, exchange=exchange)
        x = torch.from_numpy(part.x_rows).cuda()
        logits = torch.empty((pm.n_loc, pm.classes), dtype=torch.float32, device="cuda")
        for _ in range(3):
            pm.forward(x, logits, False, False)
        torch.cuda.synchronize()
        import gatb200 as G
        G.check_device()
        # pipelined host-to-host requests (three: one slot is reused) give the same logits
        xh = torch.from_numpy(part.x_rows).pin_memory()
        outs = [torch.empty((pm.n_loc, pm.classes), dtype=torch.float32).pin_memory() for _ in range(3)]
        for o in outs:
            pm.forward_async(xh, o)
        pm.join()
        torch.cuda.synchronize()
        G.check_device()
        ref = logits.cpu()
        for o in outs:
            assert torch.equal(o, ref), "forward_async differs from forward"
        n_max = int(np.diff(part.cuts).max())
        pad = torch.zeros((n_max, pm.classes), dtype=torch.float32, device="cuda")
        pad[: pm.n_loc] = logits
        full = torch.empty((world * n_max, pm.classes), dtype=torch.float32, device="cuda")
        tdist.all_gather_into_tensor(full, pad)
        torch.cuda.synchronize()
        if rank == 0:
            f = full.cpu().numpy()
            q.put(np.concatenate([f[k * n_max: k * n_max + int(part.cuts[k + 1] - part.cuts[k])]
                                  for k in range(world)]))
        pm.close()
    finally:
        tdist.destroy_process_group()


@pytest.mark.parametrize("exchange,chunks", [("p2p", 1), ("p2p", 3), ("dma", 1), ("dma", 3), ("nccl", 4)])
def test_two_gpu_partitioned_forward_matches_single_gpu(exchange, chunks):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import configs
    import gatb200 as G
    cfg = configs.make("c2")
    g = G.DeviceGraph(cfg.graph.row, cfg.graph.col)
    m = G.DeviceModel(g, [G.DeviceLayer(p) for p in cfg.model], G.PATH_STANDARD_BF16)
    logits = torch.empty((cfg.graph.n, m.classes), dtype=torch.float32, device="cuda")
    m.forward(torch.from_numpy(cfg.graph.x).cuda(), logits, False, False)
    torch.cuda.synchronize()
    want = logits.cpu().numpy()
    m.close()

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, "c2", q, exchange, chunks)) for r in range(2)]
    for p in procs:
        p.start()
    import queue
    import time
    got, deadline = None, time.time() + 240
    while got is None:
        try:
            got = q.get(timeout=2)
        except queue.Empty:
            dead = [p.exitcode for p in procs if p.exitcode not in (None, 0)]
            if dead or time.time() > deadline:
                for p in procs:
                    p.kill()
                pytest.fail(f"rank processes failed or stalled (exit codes {[p.exitcode for p in procs]})")
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    # same math per row; only the split of long rows into segments can differ
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel <= 1e-5, rel
