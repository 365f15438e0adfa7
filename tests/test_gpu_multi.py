"""Row-partitioned forward on 2 GPUs through the C ABI (gat_b200_part_model_*).

* The C++ mirror program tests/cpp/part_test.cpp, one process per rank, each
  checking its rows against the one-GPU model of the whole graph on its own
  GPU (relative L2 <= 1e-5) and its pipelined requests against its forward
  (bit for bit): P2P exchange with 1 and 3 row chunks and with either layer-2
  exchange, NCCL with 2.
* The Python binding (gatb200.Comm / PartModel) under torch.distributed, as
  bench.py drives it: the ranks' logits gathered on rank 0 against the
  one-GPU model (relative L2 <= 1e-5), with layer 2's input rows exchanged in
  the layer-1 aggregation (the default) and with H exchanged by the layer-2
  projection.

Skipped with fewer than two GPUs. NCCL's NVLink SHARP (NVLS) is off, every
wait is bounded (process-group timeout, subprocess timeouts, the peer
barrier's own bound), and a failing rank ends the test without hanging it.
"""
import os
import socket
import subprocess
import uuid
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "gat-tfs_b200"


def _gpus():
    import torch
    return torch.cuda.device_count()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def c2_files(tmp_path_factory):
    import configs
    import gatb200 as G
    d = tmp_path_factory.mktemp("c2")
    cfg = configs.make("c2")
    G.save_graph(cfg.graph, d / "c2.gatbin")
    G.save_model(cfg.model, d / "c2.gatwgt")
    return d / "c2.gatbin", d / "c2.gatwgt"


@pytest.fixture(scope="module")
def part_bin(tmp_path_factory):
    out = tmp_path_factory.mktemp("part") / "part_test"
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-Wextra", "-I", str(ROOT / "include"),
           str(ROOT / "tests" / "cpp" / "part_test.cpp"), "-L", str(PKG), "-lgat_b200", f"-Wl,-rpath,{PKG}",
           "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return out


@pytest.mark.parametrize("exchange,chunks,layer2_inputs", [(0, 1, 1), (0, 3, 1), (0, 1, 0), (1, 2, 1)])
def test_cpp_mirror_partitioned_forward(part_bin, c2_files, tmp_path, exchange, chunks, layer2_inputs):
    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    idp = tmp_path / f"nccl_id_{uuid.uuid4().hex}"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([str(part_bin), str(c2_files[0]), str(c2_files[1]), str(r), str(world), str(idp),
                               str(exchange), str(chunks), str(layer2_inputs)], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                              env=env) for r in range(world)]
    outs = []
    try:
        for p in procs:
            o, e = p.communicate(timeout=300)
            outs.append((p.returncode, o, e))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    for rc, o, e in outs:
        assert rc == 0 and "PASS" in o, o + e


def _rank_main(rank, world, port, q, exchange, chunks, layer2_inputs=True):
    import datetime
    import torch
    import torch.distributed as tdist
    import configs
    import gatb200 as G
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    tdist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                             device_id=torch.device("cuda", rank))
    try:
        uid = [G.comm_id() if rank == 0 else None]
        tdist.broadcast_object_list(uid, src=0)
        comm = G.Comm(world, rank, uid[0])
        part = configs.make_part("c2", rank, world)
        layers = [G.DeviceLayer(p) for p in part.model]
        pm = G.PartModel(comm, part.row, part.col_rows, layers, exchange, chunks, torch.cuda.current_stream())
        if exchange == G.EXCHANGE_P2P:
            pm.set_layer2_exchange(layer2_inputs)
        assert (pm.lo, pm.hi) == (part.lo, part.hi)
        x = torch.from_numpy(part.x_rows).cuda()
        logits = torch.empty((pm.n_loc, pm.classes), dtype=torch.float32, device="cuda")
        for _ in range(3):
            pm.forward(x, logits, False, False)
        torch.cuda.synchronize()
        G.check_device()
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
        comm.close()
    finally:
        tdist.destroy_process_group()


@pytest.mark.parametrize("exchange,chunks,layer2_inputs", [(0, 1, True), (0, 2, False), (1, 1, True)])
def test_python_binding_partitioned_forward(exchange, chunks, layer2_inputs):
    import torch
    import torch.multiprocessing as mp
    if _gpus() < 2:
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
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q, exchange, chunks, layer2_inputs))
             for r in range(2)]
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
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel <= 1e-5, rel
