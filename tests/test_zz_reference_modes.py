"""Reference entry points outside the timed forward, on the GPU:

- the online TFS variants of the C++ mirror (include/gat_b200_online.hpp): icpp_online,
  icpp_block and icpp_heads_hybrid with the reference's signatures
  (baseline/tfs_online/icpp_online.hpp:37-43, icpp_block.hpp:33-39,
  icpp_heads_hybrid.hpp:18-24), through tests/cpp/mirror_test.cpp --gpu-online:
  every layer against the FP64 layer at the TFS gate, the exact counters against
  what the CSR and the degree schedule determine, aggregate() + finish against
  layer(), heads_hybrid's fallback to icpp_block outside heads 8, dim 32, and
  ref_layer's R0 trace (score, max, p, den, alpha), and standard_layer with
  the lr_reordered policies (matched attention);
- gat_b200_edge_softmax, the R0 edge weights that fixed-p fixtures hold, against
  the fixture the reference itself exported (tests/golden/fixture_small_l1.gatfix);
- the driver's operator modes (bench/main.cpp:103-151): export-fixture against
  that same file, fixed-p on it with the reference's error controls, and micro;
- the adaptive experiment driver (tfs_online/adaptive_main.cpp): its smoke and a
  full run, whose exact counters pass the reference's own work identities;
- the driver's single-layer benchmark (--layer N, bench/main.cpp:166-180) on every
  path, its exported layer output against the oracle's R0 chain;
- the driver's correctness mode (bench/main.cpp:64-97): every path's stages per
  layer against R0 with the quantized and attention-reorder controls, the chains,
  the accuracy gate, and --dump-prefix;
- the reference's own boundary test (baseline/tests/boundaries.cpp), compiled
  unchanged against the C++ mirror (oracle/compat/gat.hpp) and linked with the
  library: all 64 boundary cases, the adversarial scores and the negative tests.

The kernels underneath the online variants are checked against the oracle in
test_gpu_tfs.py. This file is collected late so that a failure here leaves the
parity suites already run; it also passes when run on its own.
"""
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

import gatb200 as G

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "gat-tfs_b200"
GOLDEN = ROOT / "tests" / "golden"

pytestmark = pytest.mark.gpu


def test_online_variants_and_r0_trace(tmp_path):
    exe = tmp_path / "mirror_test"
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-Wextra", "-I", str(ROOT / "include"),
           str(ROOT / "tests" / "cpp" / "mirror_test.cpp"), "-L", str(PKG), "-lgat_b200",
           f"-Wl,-rpath,{PKG}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe), "--gpu-online", str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "MIRROR PASS online cases=16" in r.stdout and "MIRROR PASS r0_trace" in r.stdout


def test_edge_softmax_matches_reference_fixture():
    """p and den of layer 1 from the device's FP32 projection and edge softmax,
    against the GATFIX1 file the reference's export-fixture mode wrote
    (bench/main.cpp:118-121, R0's p and den of ref_fp32.cpp:7-14)."""
    import torch
    g_host = G.load_graph(GOLDEN / "fixture_small.gatbin")
    p = G.random_model(g_host.din, g_host.classes, 11)[0]
    x, pw, den = G.read_fixture(GOLDEN / "fixture_small_l1.gatfix", g_host.row, g_host.col, p)
    n, e, K, W = g_host.n, len(g_host.col), p.heads, p.width
    g = G.DeviceGraph(g_host.row, g_host.col)
    layer = G.DeviceLayer(p)
    f32 = dict(dtype=torch.float32, device="cuda")
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    ldz = G.padded_ld(W, G.F32)
    z = torch.empty((n, ldz), **f32)
    lft, rgt = torch.empty((n, K), **f32), torch.empty((n, K), **f32)
    G.projection(layer, n, xd, p.in_, G.F32, z, G.F32, ldz, lft, rgt)
    pd, dd = torch.empty((e, K), **f32), torch.empty((n, K), **f32)
    sc, md, al = torch.empty((e, K), **f32), torch.empty((n, K), **f32), torch.empty((e, K), **f32)
    G.edge_softmax(g, K, lft, rgt, pd, dd, score=sc, mx=md, alpha=al)
    torch.cuda.synchronize()
    got_p, got_den = pd.cpu().numpy(), dd.cpu().numpy()
    assert np.abs(got_p - pw).max() <= 1e-5
    assert np.abs(got_den - den).max() <= 1e-5 * np.abs(den).max()
    # the trace is self-consistent: alpha = p / den, rows of alpha sum to 1
    a = al.cpu().numpy()
    deg = np.diff(g_host.row.astype(np.int64))
    rows = np.repeat(np.arange(n), deg)
    sums = np.zeros((n, K))
    np.add.at(sums, rows, a.astype(np.float64))
    assert np.allclose(sums[deg > 0], 1.0, atol=1e-5)
    layer.close()
    g.close()


def _driver(*args):
    cli = PKG / "gat_b200_bench"
    r = subprocess.run([str(cli), *map(str, args)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    return r.stdout


def _error(out, path, stage):
    for line in out.splitlines():
        if line.startswith(f"ERROR path={path} ") and f" stage={stage} " in line:
            return {k: float(v) for k, v in (f.split("=") for f in line.split()[4:])}
    raise AssertionError(f"no ERROR line for {path} {stage}")


def test_driver_operator_modes(tmp_path):
    graph = GOLDEN / "fixture_small.gatbin"
    # export-fixture: R0's p and den of layer 1, as the reference exported them
    fix = tmp_path / "l1.gatfix"
    out = _driver("--graph", graph, "--seed", 11, "--mode", "export-fixture", "--layer", 1, "--fixture", fix)
    assert "FIXTURE saved layer=1" in out
    g = G.load_graph(graph)
    p = G.random_model(g.din, g.classes, 11)[0]
    x, pw, den = G.read_fixture(fix, g.row, g.col, p)
    x0, pw0, den0 = G.read_fixture(GOLDEN / "fixture_small_l1.gatfix", g.row, g.col, p)
    assert np.array_equal(x, x0)
    assert np.abs(pw - pw0).max() <= 1e-5 and np.abs(den - den0).max() <= 1e-5 * np.abs(den0).max()
    # fixed-p on the reference's own fixture
    out = _driver("--graph", graph, "--seed", 11, "--mode", "fixed-p", "--layer", 1, "--fixture",
                  GOLDEN / "fixture_small_l1.gatfix", "--warmups", 1, "--repeats", 3)
    emu = _error(out, "tfs_fixed_p", "vs_pX_bf16_emulation_reduction_only")
    assert emu["finite"] == 1 and emu["max_abs"] <= 2e-4 and emu["relative_l2"] <= 2e-4
    assert _error(out, "standard_fixed_p", "vs_master_fixed_p")["relative_l2"] <= 1e-2
    assert _error(out, "tfs_fixed_p", "vs_master_fixed_p")["relative_l2"] <= 3e-2
    lines = [json.loads(l) for l in out.splitlines() if l.startswith("{")]
    assert len(lines) == 6 and {l["path"] for l in lines} == {"standard_bf16", "tfs_bf16"}
    assert all(l["mode"] == "fixed-p" and l["layer"] == 1 for l in lines)
    assert any(l.startswith("FIXED_P median_standard_ms=") for l in out.splitlines())
    # micro on layer 2 (its input is the R0 chain of layer 1)
    out = _driver("--graph", graph, "--seed", 11, "--mode", "micro", "--warmups", 1, "--repeats", 3)
    names = {f.split("=")[1] for l in out.splitlines() if l.startswith("MICRO ") for f in l.split()[1:2]}
    assert {"convert_rne", "projection_bf16", "lr_reordered_bf16", "lr_reordered_fp32", "max_prescan",
            "weighted_spmm_score_exp"} <= names


def test_adaptive_driver():
    exe = PKG / "gat_b200_tfs_adaptive"
    r = subprocess.run([str(exe), "--smoke"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "SMOKE PASS cases=6" in r.stdout, r.stdout + r.stderr
    r = subprocess.run([str(exe), str(GOLDEN / "fixture_small.gatbin"), "2", "1", "2", "4"], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    out = r.stdout.splitlines()
    checks = [l for l in out if l.startswith("CHECK ")]
    assert len(checks) == 3 * 3 + 2 + 1  # chains of 3 paths, 2 layer-2 controls, the layer-3 control
    assert all(" finite=1 " in l for l in checks)
    recs = [json.loads(l) for l in out if l.startswith("{")]
    assert len(recs) == 3 * 2 * 3 and {r["path"] for r in recs} == {"B0_BF16", "HYBRID_T16_B32",
                                                                        "TFS_L12_B0_L3_MATCHED"}
    assert sum(l.startswith("PROFILE_IDENTITY ") and l.endswith("bit_fingerprint_equal=1") for l in out) == 3
    assert sum(l.startswith("ONLINE_STATS ") for l in out) == 3 and sum(l.startswith("HEAD_WORK ") for l in out) == 3
    assert sum(l.startswith("HYBRID_MIX ") for l in out) == 2  # layers 1-2; layer 3 is icpp_block
    assert out[-1].startswith("ICPP_HEADS_COMPLETE")


@pytest.mark.parametrize("path,layer,tol", [("standard_fp32", 2, 1e-4), ("standard_bf16", 2, 1e-2),
                                            ("matched_attention", 2, 1e-2), ("tfs_bf16", 1, 3e-2),
                                            ("adaptive_bf16", 1, 3e-2), ("standard_bf16", 3, 1e-2)])
def test_driver_single_layer_benchmark(tmp_path, path, layer, tol):
    import oracle as O
    graph = GOLDEN / "fixture_small.gatbin"
    dump = tmp_path / "layer.f32"
    out = _driver("--graph", graph, "--seed", 11, "--path", path, "--mode", "benchmark", "--layer", layer,
                  "--warmups", 1, "--repeats", 3, "--output", dump)
    lines = out.splitlines()
    recs = [json.loads(l) for l in lines if l.startswith("{")]
    assert len(recs) == 3 and all(r["layer"] == layer and r["path"] == path for r in recs)
    assert all(r["total_ms"] > 0 for r in recs)
    assert sum(l.startswith(f"E2E path={path} ") and f" layer={layer} " in l for l in lines) == 3
    assert any(l.startswith("SUMMARY ") for l in lines)
    g = G.load_graph(graph)
    model = G.random_model(g.din, g.classes, 11)
    ref = O.ref_chain(g.row, g.col, g.x, [(p.w, p.al, p.ar, p.heads, p.dim) for p in model])[layer - 1]["out"]
    got = np.fromfile(dump, np.float32).reshape(ref.shape)
    e = O.errors(ref, got)
    assert e["finite"] and e["relative_l2"] <= tol, e


def test_driver_correctness_mode(tmp_path):
    graph = GOLDEN / "fixture_small.gatbin"
    prefix = tmp_path / "dump"
    out = _driver("--graph", graph, "--seed", 11, "--mode", "correctness", "--max-abs", 1, "--rel-l2", "1e-2",
                  "--dump-prefix", prefix)
    errs = [l for l in out.splitlines() if l.startswith("ERROR ")]
    # per layer: 2 quantized controls, 7 + 7 + 5 + 7 path stages, 2 reorder controls; 5 chains
    assert len(errs) == 3 * 30 + 5
    assert "CORRECTNESS finite=1 accuracy_gate=PASS" in out
    recs = [json.loads(l) for l in out.splitlines() if l.startswith("{")]
    assert len(recs) == 12 and {r["mode"] for r in recs} == {"correctness"}
    # the dumped R0 trace has the reference's names and sizes, and its chain is
    # the oracle's R0 chain
    import oracle as O
    g = G.load_graph(graph)
    model = G.random_model(g.din, g.classes, 11)
    chain = O.ref_chain(g.row, g.col, g.x, [(p.w, p.al, p.ar, p.heads, p.dim) for p in model])
    assert (tmp_path / "dump_layer1_p.f32").stat().st_size == len(g.col) * 8 * 4
    for layer in (1, 2, 3):
        got = np.fromfile(tmp_path / f"dump_layer{layer}_output.f32", np.float32)
        assert np.abs(got - chain[layer - 1]["out"].ravel()).max() <= 1e-4
    ref = np.fromfile(tmp_path / "dump_model_ref_fp32.f32", np.float32)
    std = np.fromfile(tmp_path / "dump_model_standard_fp32.f32", np.float32)
    assert ref.size == g.n * g.classes and np.abs(ref - std).max() <= 1e-5
    # a gate no BF16 path can meet fails, as in the reference
    cli = PKG / "gat_b200_bench"
    r = subprocess.run([str(cli), "--graph", str(graph), "--seed", "11", "--mode", "correctness", "--max-abs", "1e-9",
                        "--rel-l2", "1e-9"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 1 and "accuracy_gate=FAIL" in r.stdout


def test_reference_boundary_test_on_the_library():
    """oracle/_ref/boundaries_on_b200 is built (make -C oracle ref) where the
    reference tree is present and travels with the build; the test reads no
    reference file at run time."""
    exe = ROOT / "oracle" / "_ref" / "boundaries_on_b200"
    if not exe.exists():
        pytest.skip("built only where the reference tree was present at build time")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr
    assert "TESTS PASS boundary_cases=64" in r.stdout
    assert r.stdout.count("BOUNDARY PASS ") == 64 and r.stdout.count("NEGATIVE PASS ") == 6
