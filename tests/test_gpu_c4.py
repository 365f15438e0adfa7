"""Parity on the headline configuration c4 (the graph bench.py times).

c4: 2,449,029 nodes, 126,167,053 edges incl. self loops, largest in-degree
17,482; 100 -> 8x32 -> 8x32 -> 1x47, BF16 with FP32 softmax state.

* Every layer of the BF16 forward on sampled rows with complete
  neighbourhoods against FP64 (tests/sampled_fp64.py): random rows, the
  degree quantiles and the 17,482-edge hub. Gate: relative L2 <= 1e-2 over
  all sampled rows (the BF16 gate against R0), <= 3e-2 for every row.
* The whole-graph BF16 logits against the FP32 device chain (pinned to R0 at
  max-abs 1e-5 on c1, smoke1024, c2 and the boundary cases), reported beside
  the reference's own B0-BF16 error on the same files
  (tests/golden/c4_reference_errors.json, made by the reference's driver).
* Where the reference's driver is built (oracle/_ref/gat_baseline), both
  device chains against the reference's B0 FP32 logits on identical
  GATBIN1 / GATWGT1 bytes: BF16 relative L2 <= 1e-2, FP32 max-abs <= 1e-5.

Set GAT_B200_PARITY_LOG to a file path to append the measured figures as JSON
lines.
"""
import json
import os
import subprocess
from pathlib import Path

import numpy as np
import pytest

import configs
import gatb200 as G
from sampled_fp64 import sampled_forward_check

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

ROOT = Path(__file__).resolve().parents[1]
REF_BIN = ROOT / "oracle" / "_ref" / "gat_baseline"
FLOOR = json.loads((ROOT / "tests" / "golden" / "c4_reference_errors.json").read_text())


def _log(rec):
    print("PARITY " + json.dumps(rec))
    path = os.environ.get("GAT_B200_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(rec) + "\n")


def _rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / np.linalg.norm(b.astype(np.float64)))


@pytest.fixture(scope="module")
def c4():
    return configs.make("c4")


@pytest.fixture(scope="module")
def chains(c4):
    """Whole-graph logits of the BF16 and FP32 device forwards."""
    import torch
    gr = c4.graph
    g = G.DeviceGraph(gr.row, gr.col)
    layers = [G.DeviceLayer(p) for p in c4.model]
    x = torch.from_numpy(gr.x).cuda()
    out = {}
    for name, path in (("bf16", G.PATH_STANDARD_BF16), ("fp32", G.PATH_STANDARD_FP32)):
        m = G.DeviceModel(g, layers, path)
        y = torch.empty((gr.n, m.classes), dtype=torch.float32, device="cuda")
        m.forward(x, y, False, False)
        torch.cuda.synchronize()
        G.check_device()
        out[name] = y.cpu().numpy()
        m.close()
        del y
    del x
    for lay in layers:
        lay.close()
    g.close()
    torch.cuda.empty_cache()
    return out


def test_c4_shape(c4):
    gr = c4.graph
    assert (gr.n, gr.e, gr.din, gr.classes) == (2_449_029, 126_167_053, 100, 47)
    assert int(np.diff(gr.row.astype(np.int64)).max()) == 17_482
    assert (FLOOR["nodes"], FLOOR["edges"]) == (gr.n, gr.e)


def test_c4_sampled_rows_fp64(dev, c4):
    r = sampled_forward_check(c4)
    _log({"test": "c4_sampled_rows_fp64", **r})
    assert r["max_degree"] == 17_482
    assert r["rel_l2"] <= 1e-2, r
    assert r["worst"][3] <= 3e-2, r


def test_c4_bf16_chain_against_fp32_chain(dev, chains):
    bf, fp = chains["bf16"], chains["fp32"]
    assert np.isfinite(bf).all() and np.isfinite(fp).all()
    rel = _rel(bf, fp)
    mx = float(np.abs(bf - fp).max())
    floor = FLOOR["reference_bf16_vs_fp32"]
    _log({"test": "c4_bf16_vs_fp32_chain", "relative_l2": rel, "max_abs": mx,
          "reference_bf16_vs_fp32": floor})
    assert rel <= 1e-2, (rel, floor)


@pytest.mark.skipif(not REF_BIN.exists(), reason="the reference's driver is not built (oracle/_ref)")
def test_c4_against_reference_fp32(dev, c4, chains, tmp_path):
    g, w, o = tmp_path / "c4.gatbin", tmp_path / "c4.gatwgt", tmp_path / "ref_fp32.f32"
    G.save_graph(c4.graph, g)
    G.save_model(c4.model, w)
    threads = max(1, min(32, os.cpu_count() or 1))
    r = subprocess.run([str(REF_BIN), "--graph", str(g), "--weights", str(w), "--path", "standard_fp32", "--mode",
                        "benchmark", "--threads", str(threads), "--warmups", "0", "--repeats", "1", "--output",
                        str(o)], capture_output=True, text=True, timeout=1500)
    assert r.returncode == 0, r.stderr[-500:]
    ref = np.fromfile(o, np.float32).reshape(c4.graph.n, c4.graph.classes)
    rec = {"test": "c4_against_reference_b0_fp32",
           "bf16": {"relative_l2": _rel(chains["bf16"], ref), "max_abs": float(np.abs(chains["bf16"] - ref).max())},
           "fp32": {"relative_l2": _rel(chains["fp32"], ref), "max_abs": float(np.abs(chains["fp32"] - ref).max())},
           "reference_bf16_vs_fp32": FLOOR["reference_bf16_vs_fp32"]}
    _log(rec)
    assert rec["bf16"]["relative_l2"] <= 1e-2, rec
    assert rec["fp32"]["max_abs"] <= 1e-5, rec
