"""The C++ mirror of the reference API (include/gat_b200.hpp), through a test
program written like the reference's boundaries.cpp (tests/cpp/mirror_test.cpp):
host-side checks here, the layer functions on the GPU."""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "gat-tfs_b200"


@pytest.fixture(scope="module")
def mirror_bin(tmp_path_factory):
    out = tmp_path_factory.mktemp("mirror") / "mirror_test"
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-Wextra", "-I", str(ROOT / "include"),
           str(ROOT / "tests" / "cpp" / "mirror_test.cpp"), "-L", str(PKG), "-lgat_b200",
           f"-Wl,-rpath,{PKG}", "-o", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    return out


# print_times' keys, in the reference's order (baseline/src/common.cpp:155-170)
PRINT_TIMES_KEYS = [
    "path", "mode", "layer", "rep", "N", "E", "D", "K", "d", "threads", "profile", "precision", "projection_ms",
    "lr_ms", "max_prescan_ms", "score_exp_aggregate_ms", "normalize_ms", "activation_ms", "convert_ms", "total_ms",
    "workspace_bytes", "static_preprocess_ms", "panel_R", "tile_rows", "score_exp_worker_ms",
    "gather_weight_convert_worker_ms", "tile_load_worker_ms", "gather_load_worker_ms",
    "p_times_x_convert_worker_ms", "weighted_spmm_worker_ms", "amx_compute_worker_ms", "tile_store_worker_ms",
    "tile_config_worker_ms", "scheduling_worker_ms", "output_write_worker_ms", "neighbor_steps", "executed_fma",
    "padding_executed_flops"]


def test_mirror_host_checks(mirror_bin, tmp_path):
    import json
    r = subprocess.run([str(mirror_bin), "--host", str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    rec = json.loads(next(l for l in r.stdout.splitlines() if l.startswith("{")))
    assert list(rec) == PRINT_TIMES_KEYS
    assert rec["projection_ms"] == 1 and rec["total_ms"] == 3 and rec["padding_executed_flops"] == 16
    assert "MIRROR PASS host" in r.stdout and r.stdout.count("MIRROR PASS rejects") == 19


@pytest.mark.gpu
def test_mirror_layer_functions_on_gpu(mirror_bin, tmp_path):
    r = subprocess.run([str(mirror_bin), "--gpu", str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "MIRROR PASS gpu cases=12" in r.stdout


def test_mirror_online_statistics_match_the_reference(mirror_bin, tmp_path):
    """The statistics the mirror fills for icpp_online, icpp_block and
    icpp_heads_hybrid with counters=true, against the Stats the reference's own code produced on
    smoke1024 (ref_dump counters; tests/golden/tfs_counters.npz): every field,
    from the Online units (which the oracle's online counters must reproduce
    for the same block size), the CSR and the degree order."""
    import numpy as np
    import gatb200 as G
    import oracle as O
    from test_oracle_golden import smoke1024_graph
    g = smoke1024_graph()
    z = np.load(ROOT / "tests" / "golden" / "tfs_counters.npz")
    perm, _ = O.degree_schedule(g.row)
    G.save_graph(g, tmp_path / "graph.gatbin")
    perm.astype(np.uint32).tofile(tmp_path / "perm.u32")
    for b in (4, 64):
        z[f"totals_b{b}"][:5].tofile(tmp_path / f"units_b{b}.u64")
    for b in (16, 32):
        ref = z[f"blockstats_b{b}"]
        # blocks, max updates, rescales, rescale events; source neighbour steps
        units = np.array([ref[0], ref[1], ref[2], ref[3], ref[18]], np.uint64)
        _, _, _, tot = O.online_counters(g.row, g.col, perm, z["left"], z["right"], 8, b)
        assert np.array_equal(tot, units), (b, tot, units)
        units.tofile(tmp_path / f"units_b{b}.u64")
    r = subprocess.run([str(mirror_bin), "--stats", str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    got = {l.split()[1]: np.array(l.split()[2:], np.uint64) for l in r.stdout.splitlines() if l.startswith("STATS ")}
    assert len(got) == 11
    for b in (4, 16, 64):
        assert np.array_equal(got[f"online{b}"], z[f"totals_b{b}"]), b
    for b in (16, 32):
        assert np.array_equal(got[f"block{b}"], z[f"blockstats_b{b}"]), b
        for t in (1, 16, 33):
            assert np.array_equal(got[f"hybrid{b}_t{t}"], z[f"hybridstats_b{b}_t{t}"]), (b, t)


def test_reference_sources_compile_against_the_mirror():
    """The reference's own boundary test compiles unchanged against the C++ mirror
    with the adapter oracle/compat/gat.hpp, so the mirror keeps every name and
    signature it uses (where the reference tree is present: the check reads its
    source, never copies it)."""
    import os
    ref = Path(os.environ.get("GAT_B200_REF") or ROOT.parent / "reference") / "baseline"
    if not (ref / "tests" / "boundaries.cpp").exists():
        pytest.skip("reference tree absent")
    cmd = ["g++", "-std=c++17", "-fopenmp", "-fsyntax-only", "-w", "-I", str(ROOT / "oracle" / "compat"),
           "-I", str(ROOT / "include"), str(ref / "tests" / "boundaries.cpp")]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
