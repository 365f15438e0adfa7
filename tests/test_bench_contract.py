"""bench.py's output contract: one JSON line with the keys the benchmark driver
reads. The reference arm (the reference's own CPU B0, built from its sources)
runs on CPU; our arm needs a GPU. Both on the tiny configuration c1."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF_BIN = ROOT / "oracle" / "_ref" / "gat_baseline"


def _bench(*args, timeout=600):
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                       timeout=timeout, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    if not REF_BIN.exists():
        d = _bench("--impl", "reference", "--config", "c1", "--steps", "1", "--warmup", "1")
        assert d["impl"] == "reference" and "unavailable" in d
        return
    d = _bench("--impl", "reference", "--config", "c1", "--steps", "2", "--warmup", "1")
    assert d["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["unit"] == "GEdges/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["e2e"] == {"value": d["value"], "unit": "GEdges/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]


def test_reference_arm_maps_no_repo_library():
    """The reference arm's process imports no binding and maps no library of
    this repository: its inputs come from gat_b200_make_inputs (host code,
    separate program) and the forward runs in the reference's binary."""
    if not REF_BIN.exists():
        pytest.skip("the reference's driver is not built (oracle/_ref)")
    code = ("import sys, runpy; sys.argv = ['bench.py', '--impl', 'reference', '--config', 'c1', '--steps', '1', "
            "'--warmup', '3']\n"
            "try:\n    runpy.run_path('bench.py', run_name='__main__')\nexcept SystemExit:\n    pass\n"
            "maps = open('/proc/self/maps').read()\n"
            "print('MAPPED', 'libgat_b200' in maps, 'gatb200' in sys.modules, 'configs' in sys.modules)")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "MAPPED False False False" in r.stdout, r.stdout[-2000:]
    d = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith("{")][0])
    assert d["steps"] == 1 and d["warmup"] == 3
    assert "physical cores" in d["cpu_baseline"]["sample"] and "NUMA" in d["config"]["placement"]


def test_reference_arm_unavailable_on_rmat():
    d = _bench("--impl", "reference", "--config", "c5", "--steps", "1", "--warmup", "1")
    assert d["impl"] == "reference" and "not run" in d["unavailable"]


@pytest.mark.gpu
def test_gpu_arm_line():
    d = _bench("--config", "c1", "--steps", "3", "--warmup", "3")
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "roofline", "e2e", "gpu_launches", "clocks"):
        assert k in d, k
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3 and d["dtype"] == "bf16"
    assert d["config"]["workload"].startswith("c1")
    rf = d["roofline"]
    for k in ("bound", "achieved", "peak", "unit", "frac", "traffic"):
        assert k in rf, k
    assert rf["bound"] == "hbm" and rf["unit"] == "GB/s" and abs(rf["frac"] - rf["achieved"] / rf["peak"]) < 1e-3
    e = d["e2e"]
    assert e["unit"] == "GEdges/s" and e["value"] > 0
    assert e["h2d_bytes_per_step"] == 1024 * 128 * 4 and e["d2h_bytes_per_step"] == 1024 * 40 * 4
    assert d["gpu_launches"] > 0
    assert {"sm_mhz", "sm_max_mhz", "reasons"} <= set(d["clocks"])
    assert "cpu_baseline" in d
    # the timed forward's own output, checked outside the timed region
    par = d["parity"]
    assert par["vs_1gpu"]["rows"] == 1024 and par["vs_1gpu"]["relative_l2"] <= 1e-5
    assert par["vs_fp64"]["relative_l2"] <= 1e-2 and par["vs_fp64"]["layer"] == 3
    assert "others" in rf and "aggregate_l3" in rf["others"]
