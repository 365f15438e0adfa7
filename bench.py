"""Three-layer GAT forward throughput on B200 (the reference's headline metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: config c4 (products-shaped seeded power-law graph, 2,449,029 nodes,
126,167,053 edges incl. self loops, 100 -> 8x32 -> 8x32 -> 1x47, BF16 with FP32
softmax state). One step = one full three-layer forward. Metric: GEdges/s =
3*E / t_forward (every layer traverses all E edges); ms_per_step is the
forward time. Prints ONE JSON line (rank 0).

  value    device-resident inputs, CUDA events on the launch stream, max over ranks
  e2e      the same forward through the C-ABI model call with pinned HOST input
           (FP32 X) and HOST logits: H2D + forward + D2H inside the timed region
  roofline the aggregation kernel (the dominant one): algorithmic bytes per
           launch / its CUDA-event duration inside the timed region vs the
           measured HBM copy bandwidth
  cpu_baseline  the reference's own B0 BF16 path (oracle/_ref/gat_baseline,
           built from the reference sources) on this host's cores, bounded sample

--impl reference times that reference CPU implementation alone on the same
workload and prints its line (rank 0 only under torchrun).

Multi-GPU: destination rows are partitioned by edge count; every layer's
projected features reach every rank's feature table through the projection
kernel's own stores over NVLink (CUDA IPC peer memory) and a cross-GPU flag
barrier (--exchange p2p, default), or through NCCL all-gathers (--exchange
nccl). NCCL otherwise only exchanges the IPC handles and runs host barriers,
so NVLink SHARP is left off (NCCL_NVLS_ENABLE=0 unless set).

--mode micro: the layer-2 micro-benchmark (config c3) on the c2 graph: input H
169,343 x 256 BF16 ~ N(0,1), W 256 x 256, a_L/a_R ~ U(-0.1, 0.1); the
reference's micro stages (bench/main.cpp:105-118) and three whole-layer
variants: transform-first (projection + fused aggregation), fixed-p
(projection + aggregation with precomputed p, bench/main.cpp:130-133) and TFS
aggregate-first; one JSON line with ms and HBM GB/s per variant.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "gat-tfs_b200"))

TMP = Path(os.environ.get("GAT_B200_TMP", "/tmp"))
REF_BIN = ROOT / "oracle" / "_ref" / "gat_baseline"
CONFIG = "c4"
# (nodes, edges) of the configurations the reference arm runs (the power-law
# and uniform ones of gat-tfs_b200/configs.py; gat_b200_make_inputs writes them)
SPECS_SHAPE = {"c1": (1024, 16384), "c2": (169_343, 2_484_941), "c4": (2_449_029, 126_167_053),
               "c4s": (612_257, 31_541_763)}
METRIC = "3-layer GAT fwd GEdges/s (2.45M nodes/126M edges, BF16)"


def metric_for(config: str, n: int, e: int) -> str:
    """BASELINE's metric for the headline configuration, the same metric on another graph otherwise."""
    return METRIC if config == CONFIG else f"3-layer GAT fwd GEdges/s ({n} nodes/{e} edges, BF16, {config})"


def graph_kind(config: str) -> str:
    import configs
    return {"powerlaw": "products-shaped power-law graph", "rmat": "RMAT(.57,.19,.19,.05) stress graph",
            "uniform": "uniform graph"}[configs.SPECS[config]["kind"]]


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default=CONFIG, choices=["c1", "c2", "c4", "c4s", "c5", "c5s"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the parity check of the timed forward's logits (printed as \"parity\")")
    ap.add_argument("--mode", choices=["forward", "micro"], default="forward")
    ap.add_argument("--path", choices=["standard", "adaptive"], default="standard",
                    help="standard: B0 on every layer; adaptive: layer 1 through TFS aggregation (tensor cores)")
    ap.add_argument("--chunks", type=int, default=1,
                    help="N>1: row chunks per rank, each projected and exchanged as soon as it is aggregated")
    ap.add_argument("--reserve-sms", type=int, default=None,
                    help="N>1, chunks>1: SMs left to each chunk's projection and exchange while the next chunk "
                         "aggregates (default 16; 0 = no overlap)")
    ap.add_argument("--layer2-exchange", choices=["inputs", "h"], default="inputs",
                    help="N>1, p2p: inputs = layer 2's input rows travel in the layer-1 aggregation's epilogue "
                         "and every rank projects the whole table; h = the layer-2 projection stores H and R "
                         "into every rank's table")
    ap.add_argument("--exchange", choices=["p2p", "nccl"], default="p2p",
                    help="N>1: p2p = the conversion / projection kernels store every rank's rows into every "
                         "rank's table over NVLink; nccl = NCCL all-gather of H and R per layer")
    return ap.parse_args()


# --------------------------------------------------------------------- clocks
class Clocks:
    """SM clock and clock-event reasons sampled every 5 ms through NVML while
    the timed region runs (read-only queries; no setting is changed). Falls
    back to nvidia-smi at 100 ms when NVML cannot be opened."""

    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap", "hw_power_brake")

    def __init__(self, device: int):
        self.device = device
        self.samples = []          # (sm_mhz, sm_max_mhz, reasons bitmask)
        self.stop_ev = threading.Event()
        self.thread = None
        self.handle = None
        self.nv = None
        try:
            import pynvml as nv
            nv.nvmlInit()
            self.nv = nv
            try:
                import torch
                pr = torch.cuda.get_device_properties(device)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                self.handle = nv.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.handle = nv.nvmlDeviceGetHandleByIndex(device)
            self.bits = {
                "hw_slowdown": nv.nvmlClocksEventReasonHwSlowdown,
                "hw_thermal_slowdown": nv.nvmlClocksEventReasonHwThermalSlowdown,
                "sw_thermal_slowdown": nv.nvmlClocksEventReasonSwThermalSlowdown,
                "sw_power_cap": nv.nvmlClocksEventReasonSwPowerCap,
                "hw_power_brake": nv.nvmlClocksEventReasonHwPowerBrakeSlowdown,
            }
        except Exception:
            self.handle = None

    def _poll(self):
        nv, h = self.nv, self.handle
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while True:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                self.samples.append((float(sm), float(mx), int(rs)))
            except Exception:
                pass
            if self.stop_ev.wait(0.005):
                break

    def start(self):
        if self.handle is None:
            self.smi = _SmiClocks(self.device)
            self.smi.start()
            return
        self.thread = threading.Thread(target=self._poll, daemon=True)
        self.thread.start()

    def stop(self) -> dict:
        if self.handle is None:
            return self.smi.stop()
        self.stop_ev.set()
        self.thread.join(timeout=5)
        sm = [s[0] for s in self.samples]
        reasons = {nm for s in self.samples for nm, bit in self.bits.items() if s[2] & bit}
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(s[1] for s in self.samples) if sm else None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvml 5 ms"}


class _SmiClocks:
    """nvidia-smi samples (every 100 ms) while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi 100 ms"}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------- reference (CPU)
MAKE_INPUTS = ROOT / "gat-tfs_b200" / "gat_b200_make_inputs"


def write_reference_inputs(config: str) -> tuple[Path, Path]:
    """GATBIN1 / GATWGT1 files of `config`, written by gat_b200_make_inputs: a
    program linked from the library's host sources only, so no process of
    the reference arm maps libgat_b200.so."""
    g = TMP / f"gat_b200_{config}.gatbin"
    w = TMP / f"gat_b200_{config}.gatwgt"
    r = subprocess.run([str(MAKE_INPUTS), config, str(g), str(w)], capture_output=True, text=True, timeout=900)
    if r.returncode != 0:
        raise RuntimeError(f"gat_b200_make_inputs {config} failed: {(r.stderr or r.stdout).strip()[-300:]}")
    return g, w


def socket_placement() -> dict:
    """One socket's physical cores (the first hardware thread of each core that
    this process may run on) and that socket's NUMA nodes: the placement of
    the reference's runs (baseline/scripts/arxiv_payload.sh:36, numactl
    --interleave over the used nodes, OMP_NUM_THREADS = physical cores)."""
    allowed = os.sched_getaffinity(0)
    rows = []
    try:
        out = subprocess.run(["lscpu", "-p=CPU,CORE,SOCKET,NODE"], capture_output=True, text=True,
                             timeout=10).stdout
        for ln in out.splitlines():
            if ln and not ln.startswith("#"):
                f = ln.split(",")
                rows.append((int(f[0]), int(f[1]), int(f[2] or 0), int(f[3] or 0)))
    except Exception:
        rows = []
    rows = [r for r in rows if r[0] in allowed]
    if not rows:
        cpus = sorted(allowed)
        return {"cpus": cpus, "socket": 0, "nodes": [0], "sockets": 1}
    sockets = sorted({r[2] for r in rows})
    sock = max(sockets, key=lambda k: (sum(1 for r in rows if r[2] == k), -k))
    first = {}
    for cpu, core, sk, node in sorted(rows):
        if sk == sock and core not in first:
            first[core] = (cpu, node)
    cpus = sorted(c for c, _ in first.values())
    nodes = sorted({nd for _, nd in first.values()})
    return {"cpus": cpus, "socket": sock, "nodes": nodes, "sockets": len(sockets)}


def _pin_and_interleave(cpus, nodes):
    """preexec_fn of the reference process: CPU affinity to `cpus` and an
    interleaved memory policy over `nodes` (set_mempolicy(MPOL_INTERLEAVE),
    what numactl --interleave does; numactl itself is not installed). Both are
    inherited across exec."""
    def fn():
        os.sched_setaffinity(0, cpus)
        try:
            import ctypes
            libc = ctypes.CDLL(None, use_errno=True)
            mask = (ctypes.c_ulong * 2)()
            for nd in nodes:
                mask[nd // 64] |= 1 << (nd % 64)
            libc.syscall(238, 3, mask, 129)  # SYS_set_mempolicy (x86-64), MPOL_INTERLEAVE
        except Exception:
            pass
    return fn


def run_reference(config: str, warmups: int, repeats: int, timeout_s: int = 1800) -> dict:
    """The reference's B0 BF16 path (baseline/bench/main.cpp benchmark mode),
    built from its sources into oracle/_ref/gat_baseline, on one socket's
    physical cores with memory interleaved over that socket's NUMA nodes."""
    if not REF_BIN.exists():
        return {"unavailable": "oracle/_ref/gat_baseline was not built (reference tree absent at build time)"}
    if not MAKE_INPUTS.exists():
        return {"unavailable": "gat-tfs_b200/gat_b200_make_inputs was not built"}
    g, w = write_reference_inputs(config)
    pl = socket_placement()
    threads = len(pl["cpus"])
    env = dict(os.environ, OMP_NUM_THREADS=str(threads), MKL_NUM_THREADS=str(threads), OMP_PROC_BIND="close",
               OMP_PLACES="cores")
    cmd = [str(REF_BIN), "--graph", str(g), "--weights", str(w), "--path", "standard_bf16", "--mode", "benchmark",
           "--threads", str(threads), "--warmups", str(warmups), "--repeats", str(repeats)]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=timeout_s,
                           preexec_fn=_pin_and_interleave(pl["cpus"], pl["nodes"]))
    except subprocess.TimeoutExpired:
        return {"unavailable": f"reference B0 run exceeded {timeout_s} s"}
    if r.returncode != 0:
        return {"unavailable": f"reference B0 exited {r.returncode}: {(r.stderr or r.stdout).strip()[-200:]}"}
    totals = [float(m) for m in re.findall(r"^E2E path=\S+ rep=\d+ layer=0 total_ms=([0-9.eE+-]+)", r.stdout, re.M)]
    if not totals:
        return {"unavailable": "no E2E lines in reference output"}
    med = statistics.median(totals)
    where = (f"socket {pl['socket']} of {pl['sockets']}: {threads} physical cores, OMP_PLACES=cores, memory "
             f"interleaved over NUMA node(s) {pl['nodes']}")
    return {"median_ms": med, "totals_ms": totals, "threads": threads, "placement": where}


# ------------------------------------------------------------------ our arm
def agg_bytes(n, e, heads, dim, out_bytes_per_elem):
    """Algorithmic bytes of one aggregation launch: rowptr, col, L of the row,
    R of every edge's source, H row of every edge's source (BF16), the output."""
    return 8 * (n + 1) + 4 * e + 4 * n * heads + 4 * e * heads + 2 * e * heads * dim + out_bytes_per_elem * n * heads * dim


def _bf16_rows(t, idx, width):
    """BF16 rows idx of device tensor t (int16 storage) as float64 (host)."""
    import numpy as np
    import torch
    import gatb200 as G
    sel = t.index_select(0, torch.from_numpy(np.asarray(idx, np.int64)).to(t.device)).cpu().numpy()
    return G.bf16_to_f32(sel.view(np.uint16)[:, :width]).astype(np.float64)


def _fp64_layer(xn, xi, w, al, ar, heads, dim):
    """Output layer of one destination row in FP64 (R0's semantics,
    baseline/src/ref_fp32.cpp:3-26, on BF16 inputs and BF16 W)."""
    import numpy as np
    z, zi = xn @ w, xi @ w
    zh = z.reshape(len(xn), heads, dim)
    L = (zi.reshape(heads, dim) * al.reshape(heads, dim)).sum(1)
    s = L[None, :] + (zh * ar.reshape(1, heads, dim)).sum(2)
    s = np.where(s > 0, s, 0.2 * s)
    p = np.exp(s - s.max(0, keepdims=True))
    return ((p / p.sum(0, keepdims=True))[:, :, None] * zh).sum(0).reshape(-1)


def parity(cfg, got, nsample=48, seed=17) -> dict:
    """Checks the logits `got` ([n, classes] FP32, host) of the forward just
    timed. The 1-GPU forward runs layer by layer (gat_b200_standard_layer,
    BF16) on the same inputs; `got` is compared with its logits over all rows
    (vs_1gpu), and on sampled rows (random ones, the 50/90/99/99.9/99.99 %
    degree quantiles and the largest hub) with an FP64 recomputation of layer
    3 from that forward's layer-3 input rows of every neighbour (vs_fp64)."""
    import numpy as np
    import torch
    import gatb200 as G
    gr = cfg.graph
    n = gr.n
    g = G.DeviceGraph(gr.row, gr.col)
    layers = [G.DeviceLayer(p) for p in cfg.model]
    try:
        ld0 = G.padded_ld(gr.din, G.BF16)
        x0 = torch.zeros((n, ld0), dtype=torch.int16, device="cuda")
        for a in range(0, n, 1 << 20):
            b = min(n, a + (1 << 20))
            G.convert(b - a, gr.din, torch.from_numpy(gr.x[a:b]).cuda(), gr.din, x0[a:b], ld0)
        ldx = G.padded_ld(256, G.BF16)
        h = torch.zeros((n, ldx), dtype=torch.int16, device="cuda")
        left = torch.zeros((n, 8), dtype=torch.float32, device="cuda")
        right = torch.zeros((n, 8), dtype=torch.float32, device="cuda")
        xs = [x0, torch.zeros((n, ldx), dtype=torch.int16, device="cuda"),
              torch.zeros((n, ldx), dtype=torch.int16, device="cuda")]
        p3 = cfg.model[2]
        ref = torch.zeros((n, p3.width), dtype=torch.float32, device="cuda")
        for l, p in enumerate(cfg.model):
            hidden = l < 2
            G.standard_layer(g, layers[l], xs[l], ld0 if l == 0 else ldx, G.PATH_STANDARD_BF16, hidden, h, left,
                             right, xs[l + 1] if hidden else ref, G.BF16 if hidden else G.F32,
                             ldx if hidden else p3.width)
        torch.cuda.synchronize()
        G.check_device()
        ref_h = ref.cpu().numpy()
        got = np.asarray(got, np.float32)
        d = got.astype(np.float64) - ref_h
        vs1 = {"relative_l2": float(np.linalg.norm(d) / np.linalg.norm(ref_h)), "max_abs": float(np.abs(d).max()),
               "rows": int(n)}
        deg = np.diff(gr.row.astype(np.int64))
        rng = np.random.default_rng(seed)
        order = np.argsort(deg, kind="stable")
        quant = [order[int(q * (n - 1))] for q in (0.5, 0.9, 0.99, 0.999, 0.9999)] + [int(order[-1])]
        rows = np.unique(np.concatenate([rng.choice(n, nsample, replace=False), quant]))
        w = G.bf16_to_f32(G.rne(p3.w)).astype(np.float64)
        al, ar = p3.al.astype(np.float64), p3.ar.astype(np.float64)
        err, nrm = 0.0, 0.0
        for i in rows:
            nb = gr.col[int(gr.row[i]):int(gr.row[i + 1])]
            want = _fp64_layer(_bf16_rows(xs[2], nb, p3.in_), _bf16_rows(xs[2], [i], p3.in_)[0], w, al, ar,
                               p3.heads, p3.dim)
            err += float(((got[i].astype(np.float64) - want) ** 2).sum())
            nrm += float((want ** 2).sum())
        vs64 = {"relative_l2": (err / nrm) ** 0.5 if nrm else 0.0, "rows": int(len(rows)),
                "largest_degree": int(deg.max()), "layer": 3}
        return {"vs_1gpu": vs1, "vs_fp64": vs64}
    finally:
        for lay in layers:
            lay.close()
        g.close()
        torch.cuda.empty_cache()


def log(msg):
    """Progress line on stderr, tagged with the rank (stdout carries only the JSON line)."""
    print(f"[bench rank {os.environ.get('RANK', '0')}] {msg}", file=sys.stderr, flush=True)



def run_micro(args) -> int:
    """Config c3: layer 2 of the c2 graph with its own seeded input and weights."""
    import numpy as np
    import torch
    import configs
    import gatb200 as G
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream()
    g_host = configs.make_graph("c2", features=False)
    n, e = g_host.n, g_host.e
    K, d, D = 8, 32, 256
    W = K * d
    hx = G.synth_normal((n, D), 303, 1)  # the layer-2 input H ~ N(0,1) (BF16 on device)
    w = G.synth_uniform((D, W), -np.sqrt(6.0 / (D + W)), np.sqrt(6.0 / (D + W)), 303, 2)
    al = G.synth_uniform((W,), -0.1, 0.1, 303, 3)
    ar = G.synth_uniform((W,), -0.1, 0.1, 303, 4)
    p = G.Param(D, K, d, w, al, ar)
    g = G.DeviceGraph(g_host.row, g_host.col, stream)
    layer = G.DeviceLayer(p)
    ld = G.padded_ld(D, G.BF16)
    xf = torch.from_numpy(hx).cuda()
    xb = torch.zeros((n, ld), dtype=torch.int16, device="cuda")
    h = torch.zeros((n, ld), dtype=torch.int16, device="cuda")
    f32 = dict(dtype=torch.float32, device="cuda")
    left, right, mx, den = (torch.empty((n, K), **f32) for _ in range(4))
    out = torch.empty((n, W), **f32)
    outb = torch.zeros((n, ld), dtype=torch.int16, device="cuda")
    G.convert(n, D, xf, D, xb, ld, stream)
    torch.cuda.synchronize()

    def t_ms(fn, k=None):
        k = k or max(3, args.steps)
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        times = []
        for _ in range(k):
            s0.record(stream)
            fn()
            s1.record(stream)
            torch.cuda.synchronize()
            times.append(s0.elapsed_time(s1))
        G.check_device()
        return statistics.median(times)

    # weights of the fixed-p variant: p = exp(leaky(L+R) - m) from this layer's L/R
    G.projection(layer, n, xb, ld, G.BF16, h, G.BF16, ld, left, right, stream)
    G.max_prescan(g, K, left, right, mx, stream)
    torch.cuda.synchronize()
    L, R, M = left.cpu().numpy(), right.cpu().numpy(), mx.cpu().numpy()
    dst = np.repeat(np.arange(n), np.diff(g_host.row.astype(np.int64)))
    s_ = L[dst] + R[g_host.col]
    pw = np.exp(np.where(s_ >= 0, s_, np.float32(0.2) * s_) - M[dst]).astype(np.float32)
    pden = np.zeros((n, K), np.float32)
    np.add.at(pden, dst, pw)
    fp, fd = torch.from_numpy(pw).cuda(), torch.from_numpy(pden).cuda()

    stages = {
        "convert_rne": t_ms(lambda: G.convert(n, D, xf, D, xb, ld, stream)),
        "projection_bf16": t_ms(lambda: G.projection(layer, n, xb, ld, G.BF16, h, G.BF16, ld, left, right, stream)),
        "lr_reordered_bf16": t_ms(lambda: G.lr_reordered(layer, n, xb, G.BF16, ld, G.LR_BF16, left, right,
                                                         stream=stream)),
        "lr_reordered_fp32": t_ms(lambda: G.lr_reordered(layer, n, xf, G.F32, D, G.LR_FP32, left, right,
                                                         stream=stream)),
        "max_prescan": t_ms(lambda: G.max_prescan(g, K, left, right, mx, stream)),
        "weighted_spmm_score_exp": t_ms(lambda: G.standard_aggregate(g, K, d, h, G.BF16, ld, left, right, out, W, den,
                                                                     stream=stream)),
    }
    G.projection(layer, n, xb, ld, G.BF16, h, G.BF16, ld, left, right, stream)

    def transform_first():
        G.projection(layer, n, xb, ld, G.BF16, h, G.BF16, ld, left, right, stream)
        G.aggregate_fused(g, K, d, h, G.BF16, ld, left, right, True, outb, G.BF16, ld, stream)

    def fixed_p():
        G.projection(layer, n, xb, ld, G.BF16, h, G.BF16, ld, left, right, stream)
        G.standard_aggregate(g, K, d, h, G.BF16, ld, left, right, out, W, den, fixed_p=fp, fixed_den=fd,
                             stream=stream)
        G.finish(n, K, d, den, True, out, W, stream)

    def tfs():
        G.lr_reordered(layer, n, xb, G.BF16, ld, G.LR_BF16, left, right, stream=stream)
        G.max_prescan(g, K, left, right, mx, stream)
        G.tfs_aggregate(g, layer, xb, ld, left, right, out, W, den, mx=mx, rounding=G.TFS_EDGE, stream=stream)
        G.finish(n, K, d, den, True, out, W, stream)

    gb = 1e9
    bytes_tf = (2 * n * D + 2 * n * W + 8 * n * K) + (8 * (n + 1) + 4 * e + 4 * n * K + 4 * e * K + 2 * e * W + 2 * n * W)
    bytes_fp = (2 * n * D + 2 * n * W + 8 * n * K) + (8 * (n + 1) + 4 * e + 4 * e * K + 2 * e * W + 4 * n * W + 4 * n * K) \
        + 8 * n * W
    bytes_tfs = (2 * n * D + 8 * n * K) + (8 * (n + 1) + 4 * e + 4 * e * K) + (8 * (n + 1) + 4 * e + 8 * n * K
                                                                                + 4 * e * K + 2 * e * D + 4 * n * W + 4 * n * K) + 8 * n * W
    variants = {}
    for name, fn, b, note in (("transform_first", transform_first, bytes_tf,
                               "tcgen05 projection + fused edge-softmax aggregation (BF16 out)"),
                              ("fixed_p", fixed_p, bytes_fp, "projection + aggregation with precomputed p + finish"),
                              ("tfs_aggregate_first", tfs, bytes_tfs,
                               "lr_reordered + max prescan + TFS B1 aggregation (CUDA cores: the tensor-core "
                               "TFS kernel takes inputs of at most 120 features) + finish")):
        ms = t_ms(fn)
        variants[name] = {"ms": round(ms, 4), "algorithmic_bytes": int(b), "gbs": round(b / (ms * 1e-3) / gb, 1),
                          "what": note}
    peak, peak_kind = peaks()
    line = {"metric": "layer-2 micro-benchmark (c3) ms", "unit": "ms", "higher_is_better": False,
            "mode": "micro", "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"c3: layer 2 of c2 (N={n}, E={e}), H {n}x{D} BF16 ~ N(0,1), W {D}x{W}, "
                                   "a_L/a_R ~ U(-0.1,0.1)"},
            "stages_ms": {k: round(v, 4) for k, v in stages.items()},
            "variants": variants, "hbm_peak_gbs": peak, "peak_kind": peak_kind}
    print(json.dumps(line))
    layer.close()
    g.close()
    return 0

def main():
    args = parse()
    if args.mode == "micro":
        return run_micro(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        # Rank 0 alone times the reference CPU implementation; the others exit.
        # This process never imports the library: the input files come from
        # gat_b200_make_inputs (host code only) and the timed forward runs in
        # the reference's own binary.
        if rank != 0:
            return 0
        spec = SPECS_SHAPE.get(args.config)
        if spec is None:
            print(json.dumps({"impl": "reference", "unavailable": "not run on the RMAT stress graph: the "
                              "reference's B0 keeps three FP32 workspaces of it (tens of GB) and takes minutes "
                              "per forward on the host cores"}))
            return 0
        n_, e_ = spec
        w = max(args.warmup, 3)
        k = args.steps
        res = run_reference(args.config, w, k)
        e3 = 3 * e_
        if "unavailable" in res:
            print(json.dumps({"impl": "reference", "unavailable": res["unavailable"]}))
            return 0
        v = e3 / (res["median_ms"] * 1e-3) / 1e9
        sample = (f"full {args.config} forward per step, median of {len(res['totals_ms'])} timed forwards "
                  f"after {w} warm-up; {res['placement']}")
        line = {"impl": "reference", "metric": metric_for(args.config, n_, e_),
                "value": round(v, 5), "unit": "GEdges/s", "n_gpus": 0,
                "steps": len(res["totals_ms"]), "warmup": w, "ms_per_step": round(res["median_ms"], 3),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic", "config": {"workload": args.config, "path": "reference B0 standard_bf16 (CPU)",
                                                "placement": res["placement"]},
                "cpu_baseline": {"value": round(v, 5), "unit": "GEdges/s", "cores": res["threads"],
                                 "kind": "reference", "sample": sample},
                "e2e": {"value": round(v, 5), "unit": "GEdges/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return 0

    import configs
    import numpy as np
    import torch
    import gatb200 as G

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        log("process group ready")
    stream = torch.cuda.current_stream()
    warm = max(args.warmup, 3)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(step, k):
        """ms per step of k calls of step(), CUDA events on the launch stream, max over ranks."""
        barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(k):
            step()
        t1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(t0.elapsed_time(t1) / k)

    if world == 1:
        # ---- one GPU: the C-ABI three-layer model ----
        cfg = configs.make(args.config)
        n, e, din = cfg.graph.n, cfg.graph.e, cfg.graph.din
        n_loc, e_loc = n, e
        g = G.DeviceGraph(cfg.graph.row, cfg.graph.col, stream)
        layers = [G.DeviceLayer(p) for p in cfg.model]
        model = G.DeviceModel(g, layers, G.PATH_ADAPTIVE_BF16 if args.path == "adaptive" else G.PATH_STANDARD_BF16)
        classes = model.classes
        x_rows = cfg.graph.x
        x_dev = torch.from_numpy(x_rows).cuda()
        logits = torch.empty((n, classes), dtype=torch.float32, device="cuda")
        fwd = lambda x, y, xh, yh: model.forward(x, y, xh, yh, stream)
        for _ in range(warm):
            fwd(x_dev, logits, False, False)
        torch.cuda.synchronize()
        G.check_device()
        model.enable_timing(args.steps)
        clocks = Clocks(local)
        clocks.start()
        ms = timed(lambda: fwd(x_dev, logits, False, False), args.steps)
        clk = clocks.stop()
        G.check_device()
        st = model.stage_times()
        stage_ms = {k: float(st[:, i].mean()) for i, k in enumerate(G.DeviceModel.STAGES) if k not in ("h2d", "d2h")}
        launches = model.launches()
        model.enable_timing(0)
        parallelism = "single"
    else:
        # ---- N GPUs: the C-ABI partitioned model (gat_b200_part_model_*) ----
        log("building rank-local inputs")
        part = configs.make_part(args.config, rank, world)
        log(f"rows [{part.lo}, {part.hi}) of {len(part.row) - 1}")
        n, e, din = len(part.row) - 1, part.e, part.din
        uid = [G.comm_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = G.Comm(world, rank, uid[0])
        part_layers = [G.DeviceLayer(p) for p in part.model]
        exch = G.EXCHANGE_P2P if args.exchange == "p2p" else G.EXCHANGE_NCCL
        pm = G.PartModel(comm, part.row, part.col_rows, part_layers, exch, args.chunks, stream)
        if args.reserve_sms is not None:
            pm.set_overlap(args.reserve_sms)
        if args.exchange == "p2p" and args.layer2_exchange == "h":
            pm.set_layer2_exchange(False)
        log("device model ready")
        n_loc, e_loc = pm.n_loc, pm.e_loc
        classes = pm.classes
        x_rows = part.x_rows
        x_dev = torch.from_numpy(x_rows).cuda()
        logits = torch.empty((n_loc, classes), dtype=torch.float32, device="cuda")
        fwd = lambda x, y, xh, yh: pm.forward(x, y, xh, yh, stream)
        for _ in range(warm):
            fwd(x_dev, logits, False, False)
        torch.cuda.synchronize()
        G.check_device()
        log("warm-up done")
        pm.enable_timing(True)
        clocks = Clocks(local)
        clocks.start()
        ms = timed(lambda: fwd(x_dev, logits, False, False), args.steps)
        clk = clocks.stop()
        G.check_device()
        stage_ms = pm.stage_times()  # last timed step
        pm.enable_timing(False)
        launches = pm.launches()
        if args.exchange == "p2p":
            l2 = ("layer 2: the layer-1 aggregation stores every output row into every rank's layer-2 input "
                  "table and each rank projects the whole table; layer 3"
                  if args.layer2_exchange == "inputs" else "layers 2-3")
            how = ("layer 1: the conversion kernel stores every input row into every rank's input table over "
                   "NVLink (CUDA IPC peer memory) and each rank projects the whole table; " + l2 +
                   ": the projection kernel stores each H/R tile into every rank's table; a cross-GPU flag "
                   "barrier closes each exchange")
        else:
            how = "NCCL all-gather of each layer's H and R"
        if args.chunks > 1 and args.exchange == "p2p" and args.reserve_sms != 0:
            how += (f"; chunk c's projection and exchange overlap chunk c+1's aggregation on "
                    f"{16 if args.reserve_sms is None else args.reserve_sms} reserved SMs")
        parallelism = (f"rows{world}: destination rows split by edge count, {args.chunks} row chunk(s) per "
                       f"rank; {how}")

    # roofline of the dominant kernel: the hidden-layer aggregation (agg_kernel,
    # launches of layers 1 and 2, the same bytes each), averaged over the timed
    # steps. Layer 3's aggregation and the projections are reported beside it.
    # Under the multi-GPU pipeline with the layer-2 input exchange, layer 1's
    # aggregation also stores every output row to the peers, so layer 2's launch
    # alone is the kernel's figure; with chunks > 1 a layer's time also holds the
    # projections of its earlier chunks, and the figure is a lower bound.
    peak, peak_kind = peaks()
    b_hid = agg_bytes(n_loc, e_loc, 8, 32, 2)
    b_l3 = agg_bytes(n_loc, e_loc, 1, classes, 4)
    x2_inputs = world > 1 and args.exchange == "p2p" and args.layer2_exchange == "inputs"
    if (world == 1 and args.path == "adaptive") or x2_inputs:
        hid = [stage_ms["aggregate_l2"]]
    else:
        hid = [stage_ms["aggregate_l1"], stage_ms["aggregate_l2"]]
    l3_ms = stage_ms["aggregate_l3"]
    hid_ms = sum(hid) / len(hid)
    achieved = b_hid / (hid_ms * 1e-3) / 1e9
    traffic = None
    prof = ROOT / "profiles" / "aggregate_c4_traffic.json"
    if prof.exists() and world == 1 and args.config == "c4" and args.path == "standard":
        pl = json.loads(prof.read_text())["per_launch_bytes"]
        traffic = (pl["layer1"] + pl["layer2"]) / 2
    others = {"aggregate_l3": {"ms": round(l3_ms, 4), "algorithmic_bytes": int(b_l3),
                               "achieved_gbs": round(b_l3 / (l3_ms * 1e-3) / 1e9, 1),
                               "frac": round(b_l3 / (l3_ms * 1e-3) / 1e9 / peak, 4)}}
    if world == 1:
        # (N > 1: the projection stages also hold the exchange; stage_ms lists them)
        widths = [(din, 8, 32), (256, 8, 32), (256, 1, classes)]
        for l, (D, K, dd) in enumerate(widths, 1):
            pb = 2 * n_loc * D + 2 * D * (K * dd + 2 * K) + 2 * n_loc * K * dd + 8 * n_loc * K
            pms = stage_ms[f"projection_l{l}"]
            others[f"projection_l{l}"] = {"ms": round(pms, 4), "algorithmic_bytes": int(pb),
                                          "achieved_gbs": round(pb / (pms * 1e-3) / 1e9, 1),
                                          "frac": round(pb / (pms * 1e-3) / 1e9 / peak, 4)}

    # e2e: the same forward with pinned HOST input rows and HOST logits, through the C ABI.
    # Latency: one synchronous call per step (upload, forward, download, wait).
    x_host = torch.from_numpy(x_rows).pin_memory()
    l_host = [torch.empty((n_loc, classes), dtype=torch.float32).pin_memory() for _ in range(2)]

    def e2e_step():
        fwd(x_host, l_host[0], True, True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    e2e_sync_ms = timed(e2e_step, max(1, min(args.steps, 5)))
    # Throughput: a stream of requests through gat_b200_model_forward_async, where request
    # k's download and request k+1's upload overlap compute (one GPU only).
    k_pipe = max(2, min(args.steps, 20))
    if world == 1:
        submit = lambda i: model.forward_async(x_host, l_host[i & 1], stream)
        join = lambda: model.join(stream)
        api = "gat_b200_model_forward_async"
    else:
        submit = lambda i: pm.forward_async(x_host, l_host[i & 1], stream)
        join = lambda: pm.join(stream)
        api = "gat_b200_part_model_forward_async on every rank (its rows of X up, its logits down)"
    for i in range(2):
        submit(i)
    join()
    torch.cuda.synchronize()

    def pipe_steps():
        for i in range(k_pipe):
            submit(i)
        join()

    e2e_ms = timed(pipe_steps, 1) / k_pipe
    G.check_device()
    e2e_mode = (f"pipelined: {k_pipe} requests through {api}, each uploading X and downloading logits "
                "(pinned host buffers); request k's download and k+1's upload overlap compute")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config.startswith("c5"):
        cpu = {"value": None, "unit": "GEdges/s", "cores": len(socket_placement()["cpus"]), "kind": "reference",
               "sample": "not run: the reference's B0 keeps three FP32 workspaces of the RMAT graph "
                         "(tens of GB) and takes minutes per forward on the host cores"}
    elif rank == 0 and world == 1 and not args.no_cpu_baseline:
        res = run_reference(args.config, 1, 2)
        if "unavailable" in res:
            cpu = {"value": None, "unit": "GEdges/s", "cores": len(socket_placement()["cpus"]), "kind": "reference",
                   "sample": res["unavailable"]}
        else:
            cpu = {"value": round(3 * e / (res["median_ms"] * 1e-3) / 1e9, 5), "unit": "GEdges/s",
                   "cores": res["threads"], "kind": "reference",
                   "sample": f"full {args.config} forward, median of {len(res['totals_ms'])} after 1 warm-up "
                             f"(reference B0 standard_bf16, {res['median_ms']:.1f} ms; {res['placement']})"}

    # parity of the timed forward's logits (outside every timed region): rank 0
    # gathers all ranks' rows, then checks them after the process group is gone
    got = None
    if world == 1:
        got = logits.cpu().numpy()
    else:
        n_max = int(np.diff(part.cuts).max())
        pad = torch.zeros((n_max, classes), dtype=torch.float32, device="cuda")
        pad[:n_loc] = logits
        full = torch.empty((world * n_max, classes), dtype=torch.float32, device="cuda")
        dist.all_gather_into_tensor(full, pad)
        if rank == 0:
            fh = full.cpu().numpy()
            got = np.concatenate([fh[k * n_max:k * n_max + int(part.cuts[k + 1] - part.cuts[k])]
                                  for k in range(world)])
        del full, pad
        # every rank's stage times of its last timed step (rank balance)
        names = list(stage_ms)
        mine = torch.tensor([float(stage_ms[k]) for k in names], dtype=torch.float32, device="cuda")
        allst = torch.empty(world * len(names), dtype=torch.float32, device="cuda")
        dist.all_gather_into_tensor(allst, mine)
        allst = allst.view(world, len(names))
        stage_ranks = {k: [round(float(v), 4) for v in allst[:, i].tolist()] for i, k in enumerate(names)}

    line = None
    if rank == 0:
        value = 3 * e / (ms * 1e-3) / 1e9
        line = {
            "metric": metric_for(args.config, n, e), "value": round(value, 4), "unit": "GEdges/s",
            "n_gpus": world, "steps": args.steps,
            "warmup": warm, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{args.config}: {graph_kind(args.config)}, N={n}, E={e}, "
                                   f"{din}->8x32->8x32->1x{classes}",
                       "nodes": n, "edges": e,
                       "l2": f"inputs larger than L2 (H is {n * 512 / 1e9:.2f} GB per layer)",
                       "parallelism": parallelism, "path": args.path if world == 1 else "standard"},
            "stage_ms": {k: round(float(v), 4) for k, v in stage_ms.items()},
            **({"stage_ms_by_rank": stage_ranks} if world > 1 else {}),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "peak_kind": peak_kind,
                         "kernel": "agg_kernel, hidden layers (" + ("layer 2" if len(hid) == 1 else "layers 1-2") +
                                   (", rank 0 rows, last timed step" + (")" if args.chunks == 1 else
                                                                         ", incl. interleaved projections)")
                                    if world > 1 else ", mean launch over the timed steps)"),
                         "algorithmic_bytes_per_launch": int(b_hid), "others": others,
                         "dram_frac": (round(traffic / (hid_ms * 1e-3) / 1e9 / peak, 4) if traffic else None),
                         "note": "frac counts every edge's row gather as HBM traffic (the L2 serves repeat "
                                 "gathers of popular sources, so it can exceed 1); dram_frac uses the ncu DRAM "
                                 "bytes of the same launch (profiles/aggregate_c4_traffic.json)"},
            "e2e": {"value": round(3 * e / (e2e_ms * 1e-3) / 1e9, 4), "unit": "GEdges/s",
                    "ms_per_step": round(e2e_ms, 3), "mode": e2e_mode,
                    "sync_ms_per_step": round(e2e_sync_ms, 3), "h2d_bytes_per_step": n * din * 4,
                    "d2h_bytes_per_step": n * classes * 4},
            "gpu_launches": launches * args.steps,
            "clocks": clk,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
    if world == 1:
        model.close()
    else:
        pm.close()
        for lay in part_layers:
            lay.close()
        comm.close()
        dist.destroy_process_group()
    if rank == 0:
        if args.path == "standard" and not args.no_parity:
            log("parity check")
            full_cfg = cfg if world == 1 else configs.make(args.config)
            line["parity"] = parity(full_cfg, got)
        print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
