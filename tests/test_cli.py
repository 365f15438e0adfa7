"""The C++ driver gat-tfs_b200/gat_b200_bench: the reference's bench/main.cpp
interface (arguments, log lines, JSON keys of print_times, common.cpp:155-170)
over the C ABI."""
import json
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CLI = ROOT / "gat-tfs_b200" / "gat_b200_bench"
GOLDEN = ROOT / "tests" / "golden"

# the per-layer keys of the reference's print_times that its summaries read
TIMES_KEYS = ["path", "mode", "layer", "rep", "N", "E", "D", "K", "d", "threads", "profile", "precision",
              "projection_ms", "lr_ms", "max_prescan_ms", "score_exp_aggregate_ms", "normalize_ms", "activation_ms",
              "convert_ms", "total_ms", "workspace_bytes", "static_preprocess_ms", "panel_R", "tile_rows",
              "neighbor_steps", "executed_fma", "padding_executed_flops"]


def run(*args, timeout=300):
    if not CLI.exists():
        subprocess.run(["python", str(ROOT / "gat-tfs_b200" / "build.py")], check=True)
    return subprocess.run([str(CLI), *args], capture_output=True, text=True, timeout=timeout)


def test_cli_argument_errors():
    r = run("--graph")
    assert r.returncode == 1 and "FAIL arguments must be --key value" in r.stderr
    r = run("--graph", "x", "--graph", "y")
    assert r.returncode == 1 and "FAIL duplicate argument: --graph" in r.stderr
    r = run("--graph", "x", "--nope", "1")
    assert r.returncode == 1 and "FAIL unknown option: --nope" in r.stderr
    r = run("--mode", "benchmark")
    assert r.returncode == 1 and "FAIL --graph is required" in r.stderr
    r = run("--graph", str(GOLDEN / "fixture_small.gatbin"), "--path", "nope")
    assert r.returncode == 1 and "FAIL bad path" in r.stderr
    r = run("--graph", str(GOLDEN / "fixture_small.gatbin"))
    assert r.returncode == 1 and "provide --weights checkpoint.bin or explicit --seed" in r.stderr
    r = run("--graph", "/nonexistent.gatbin", "--seed", "11")
    assert r.returncode == 1 and "FAIL cannot open graph" in r.stderr
    # modes and their checks (bench/main.cpp:33-35,103-121,145-147)
    g0 = str(GOLDEN / "fixture_small.gatbin")
    for args, msg in ((("--mode", "nope"), "FAIL bad mode"),
                      (("--mode", "profile"), "FAIL profile requires profile binary"),
                      (("--mode", "export-fixture"), "FAIL --fixture output is required"),
                      (("--init-policy", "cold"), "FAIL bad init policy"),
                      (("--mode", "benchmark", "--layer", "4"), "FAIL invalid benchmark controls")):
        r = run("--graph", g0, "--seed", "11", *args)
        assert r.returncode == 1 and msg in r.stderr, (args, r.stderr)
    # bench/main.cpp:61-63: the LR policy checks
    g = str(GOLDEN / "fixture_small.gatbin")
    r = run("--graph", g, "--seed", "11", "--lr-policy", "nope")
    assert r.returncode == 1 and "FAIL bad LR policy" in r.stderr
    r = run("--graph", g, "--seed", "11", "--path", "tfs_bf16", "--lr-policy", "z_avx")
    assert r.returncode == 1 and "FAIL reordered LR path requires bf16/fp32/avx" in r.stderr
    r = run("--graph", g, "--seed", "11", "--path", "matched_attention", "--lr-policy", "fp32")
    assert r.returncode == 1 and "not available for path matched_attention" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("path", ["standard_bf16", "standard_fp32", "tfs_bf16", "matched_attention", "adaptive_bf16"])
def test_cli_benchmark_log_lines(path):
    r = run("--graph", str(GOLDEN / "fixture_small.gatbin"), "--seed", "11", "--path", path, "--mode",
            "benchmark", "--repeats", "2", "--warmups", "1")
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    for tag in ("ENV ", "STATIC ", "CONFIG ", "MODEL ", "COLD ", "E2E ", "SUMMARY "):
        assert any(ln.startswith(tag) for ln in lines), tag
    recs = [json.loads(ln) for ln in lines if ln.startswith("{")]
    assert len(recs) == 2 * 3
    for rec in recs:
        for k in TIMES_KEYS:
            assert k in rec, k
        assert rec["path"] == path and rec["N"] == 200 and rec["total_ms"] >= 0


# ---- gat_b200_tfs_online: the reference's tfs_online/main.cpp interface -------
ONLINE = ROOT / "gat-tfs_b200" / "gat_b200_tfs_online"


def run_online(*args, timeout=300):
    if not ONLINE.exists():
        subprocess.run(["python", str(ROOT / "gat-tfs_b200" / "build.py")], check=True)
    return subprocess.run([str(ONLINE), *args], capture_output=True, text=True, timeout=timeout)


def test_tfs_online_argument_errors():
    r = run_online("a", "b")
    assert r.returncode == 1 and "ICPP_ONLINE_FAIL usage: icpp_online GRAPH THREADS" in r.stderr
    r = run_online("g", "0", "1", "1", "16", "1")
    assert r.returncode == 1 and "ICPP_ONLINE_FAIL invalid config" in r.stderr
    r = run_online("g", "2", "1", "1", "16,65", "1")
    assert r.returncode == 1 and "ICPP_ONLINE_FAIL invalid block" in r.stderr
    r = run_online("g", "2", "1", "1", "", "1")
    assert r.returncode == 1 and "ICPP_ONLINE_FAIL no Online path" in r.stderr


@pytest.mark.gpu
def test_tfs_online_smoke_and_report():
    r = run_online("--smoke")
    assert r.returncode == 0 and "SMOKE PASS cases=8" in r.stdout, r.stdout + r.stderr
    r = run_online(str(GOLDEN / "fixture_small.gatbin"), "4", "0", "1", "16,64", "1")
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.splitlines()
    tags = [ln.split(" ", 1)[0] for ln in lines]
    assert tags.count("CONFIG") == 1 and tags.count("STATIC") == 3
    assert tags.count("CHECK") == 3 * 4 + 5 * 3  # common-input controls + every path's chain
    assert tags.count("ORACLE_COVERAGE") == 3
    assert tags.count("PROFILE_IDENTITY") == 6 and tags.count("ONLINE_STATS") == 6
    assert all("bit_fingerprint_equal=1" in ln for ln in lines if ln.startswith("PROFILE_IDENTITY"))
    recs = [json.loads(ln) for ln in lines if ln.startswith("{")]
    assert len(recs) == 5 * 3 and {r_["path"] for r_ in recs} == {"B0_FP32", "B0_BF16", "B1_TFS_PREMAX",
                                                                 "ICPP_TFS_ONLINE_B16", "ICPP_TFS_ONLINE_B64"}
    # online vs B1 on a common input: only rescale roundings apart
    for ln in lines:
        if ln.startswith("CHECK") and "B1_PREMAX_same_input_same_LR" in ln:
            assert "original_abs_003_gate=PASS" in ln, ln
    assert lines[-1].startswith("ICPP_ONLINE_COMPLETE")


# ---- gat_b200_tfs_adaptive: the reference's tfs_online/adaptive_main.cpp interface ----
ADAPTIVE = ROOT / "gat-tfs_b200" / "gat_b200_tfs_adaptive"


def test_tfs_adaptive_argument_errors():
    if not ADAPTIVE.exists():
        subprocess.run(["python", str(ROOT / "gat-tfs_b200" / "build.py")], check=True)
    r = subprocess.run([str(ADAPTIVE), "a", "b"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "ICPP_HEADS_FAIL usage: icpp_heads GRAPH THREADS" in r.stderr
    r = subprocess.run([str(ADAPTIVE), "g", "0", "1", "1", "1"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "ICPP_HEADS_FAIL invalid configuration" in r.stderr


@pytest.mark.parametrize("config", ["c1", "c2"])
def test_make_inputs_equals_binding(config, tmp_path):
    """gat_b200_make_inputs (host objects only, used by the CPU reference arm)
    writes the same GATBIN1 / GATWGT1 bytes as configs.make + the binding."""
    import configs
    import gatb200 as G
    exe = ROOT / "gat-tfs_b200" / "gat_b200_make_inputs"
    r = subprocess.run([str(exe), config, str(tmp_path / "a.gatbin"), str(tmp_path / "a.gatwgt")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith(f"INPUTS config={config} ")
    c = configs.make(config)
    G.save_graph(c.graph, tmp_path / "b.gatbin")
    G.save_model(c.model, tmp_path / "b.gatwgt")
    for ext in ("gatbin", "gatwgt"):
        assert (tmp_path / f"a.{ext}").read_bytes() == (tmp_path / f"b.{ext}").read_bytes(), ext
    # the RMAT configurations are generated on the GPU only: refused
    assert subprocess.run([str(exe), "c5", "x", "y"], capture_output=True, text=True).returncode == 1
