"""Regenerates the golden fixtures in tests/golden/ from the reference itself.

Run where the reference source tree exists (its location in the GAT_B200_REF
environment variable, or a `reference` directory next to this repository)
after `make -C oracle all ref`:

    python tests/golden/make_golden.py

What it records (all produced by the reference's own code, compiled from its
sources in place by oracle/Makefile; nothing here is hand-written):
  * smoke1024.gatbin: the reference's committed test graph
    (implementation/data/smoke1024.gatbin). It is regenerated here with the
    reference's own algorithm (implementation/tools/prepare_smoke.py:9-23,
    numpy default_rng(20260928)) and must hash to the committed file.
  * smoke1024_seed11.npz: R0 three-layer chain on smoke1024 with the
    reference's random_model(seed 11): per-layer left/right/max/den, final
    logits, B0 BF16 / FP32 chain logits, degree_schedule perm and
    neighbor_steps, and the hash of the GATWGT1 file the reference saved.
  * config1.npz: the same dumps for the c1 graph and Glorot weights produced
    by this repository's generator (GATBIN1 / GATWGT1 hashes recorded).
  * boundary.npz: R0 (and for a subset B0 BF16) outputs of the 64 D/K/d
    cases of baseline/tests/boundaries.cpp, plus its degree schedule.
  * tfs.npz: the TFS aggregation family on a subset of the boundary cases:
    B1 tfs_aggregate, icpp_online (block 16), icpp_block (block 32) and
    icpp_heads_hybrid (block 32, threshold 16) outputs, with the inputs the
    reference computed for them (BF16- and FP32-policy L/R, prescan max, blr).
    The chain npz files also hold the tfs_bf16 path's three-layer logits.
  * tfs_counters.npz: icpp_online's exact counters (icpp_online.hpp:18-22) on
    smoke1024 with attention scores rising with the source id, for neighbour
    blocks of 4, 16 and 64: per (row, head) blocks / max updates / rescales
    and the Stats totals, with the L/R the reference used; and on the same
    inputs icpp_block's statistics (blocks of 16 and 32) and
    icpp_heads_hybrid's (blocks of 16 and 32, thresholds 1, 16 and 33).
  * fixture_small_l1.gatfix (+ fixture_small.gatbin): a GATFIX1 fixed-p
    fixture written by the reference's own export-fixture mode
    (bench/main.cpp:103-116) for layer 1 of random_model(seed 11) on a small
    seeded uniform graph from this repository's generator.
"""
import hashlib
import json
import os
import struct
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "gat-tfs_b200"))
import configs  # noqa: E402
import gatb200 as G  # noqa: E402

REF = Path(os.environ.get("GAT_B200_REF") or ROOT.parent / "reference")
OUT = Path(__file__).resolve().parent
DUMP = ROOT / "oracle" / "_ref" / "ref_dump"


# Boundary shapes (D, K, d) kept for the TFS fixtures: the layer shapes of the
# configs (128->8x32, 256->8x32, 256->1x47) and three odd ones.
TFS_CASES = [(17, 1, 7), (33, 2, 40), (128, 8, 32), (256, 8, 32), (256, 1, 47), (128, 4, 47)]


def small_fixture_graph():
    """200 rows, 7 uniform sources + self loop, 24 features, 5 classes (seed 21)."""
    n, din, classes = 200, 24, 5
    row, col = G.synth_uniform_graph(n, 7, 21)
    x = G.synth_normal((n, din), 21, 1)
    return G.Graph(n=n, e=len(col), din=din, classes=classes, row=row, col=col, x=x)


def sha256(path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def write_smoke1024(path: Path):
    """Same draws, in the same order, as implementation/tools/prepare_smoke.py:9-23."""
    rng = np.random.default_rng(20260928)
    n, d, c = 1024, 128, 40
    degrees = [1, 2, 7, 15, 16, 17, 31, 32, 33, 63, 64, 65, 96, 127]
    row, col = [0], []
    for i in range(n):
        deg = degrees[i % len(degrees)]
        neighbors = rng.choice(n, size=deg - 1, replace=False).astype(np.uint32).tolist()
        col.extend([i] + neighbors)
        row.append(len(col))
    x = rng.normal(0, 0.5, size=(n, d)).astype("<f4")
    with path.open("wb") as f:
        f.write(struct.pack("<8sQQII", b"GATBIN1\0", n, len(col), d, c))
        np.asarray(row, dtype="<u8").tofile(f)
        np.asarray(col, dtype="<u4").tofile(f)
        x.tofile(f)


def load(d: Path, name: str, dtype=np.float32):
    return np.fromfile(d / name, dtype=dtype)


def chain_npz(d: Path, n: int, classes: int) -> dict:
    out = dict(perm=load(d, "perm.u32", np.uint32), steps=load(d, "steps.u64", np.uint64))
    for l, k in ((1, 8), (2, 8), (3, 1)):
        for s in ("left", "right", "max", "den"):
            out[f"ref_l{l}_{s}"] = load(d, f"ref_l{l}_{s}.f32").reshape(n, k)
    out["ref_logits"] = load(d, "ref_l3_out.f32").reshape(n, classes)
    out["b0bf16_logits"] = load(d, "b0bf16_out.f32").reshape(n, classes)
    out["b0fp32_logits"] = load(d, "b0fp32_out.f32").reshape(n, classes)
    out["tfsbf16_logits"] = load(d, "tfsbf16_out.f32").reshape(n, classes)
    return out


def main():
    if not DUMP.exists():
        sys.exit("build the reference harness first: make -C oracle all ref")
    manifest = {}
    with tempfile.TemporaryDirectory() as tmp:
        tmp = Path(tmp)
        # smoke1024
        smoke = tmp / "smoke1024.gatbin"
        write_smoke1024(smoke)
        manifest["smoke1024_gatbin_sha256"] = sha256(smoke)
        ref_file = REF / "implementation" / "data" / "smoke1024.gatbin"
        if ref_file.exists():
            assert sha256(ref_file) == manifest["smoke1024_gatbin_sha256"], "smoke1024 regeneration differs"
            manifest["smoke1024_matches_reference_file"] = True
        d = tmp / "smoke"
        d.mkdir()
        subprocess.run([str(DUMP), "chain", str(smoke), "seed:11", str(d)], check=True)
        manifest["smoke1024_seed11_gatwgt_sha256"] = sha256(d / "weights.gatwgt")
        np.savez_compressed(OUT / "smoke1024_seed11.npz", **chain_npz(d, 1024, 40))

        # icpp_online's exact counters on smoke1024 (ref_dump counters)
        d = tmp / "counters"
        d.mkdir()
        subprocess.run([str(DUMP), "counters", str(smoke), str(d)], check=True)
        c = {"left": load(d, "counters_left.f32").reshape(1024, 8),
             "right": load(d, "counters_right.f32").reshape(1024, 8)}
        for b in (4, 16, 64):
            for name in ("rowblocks", "rowupdates", "rowrescales"):
                c[f"{name}_b{b}"] = np.fromfile(d / f"counters_b{b}_{name}.u64", np.uint64).reshape(1024, 8)
            c[f"totals_b{b}"] = np.fromfile(d / f"counters_b{b}_totals.u64", np.uint64)
        # icpp_block's and icpp_heads_hybrid's statistics on the same inputs
        for b in (16, 32):
            c[f"blockstats_b{b}"] = np.fromfile(d / f"counters_block{b}_stats.u64", np.uint64)
            for t in (1, 16, 33):
                c[f"hybridstats_b{b}_t{t}"] = np.fromfile(d / f"counters_hybrid{b}_t{t}_stats.u64", np.uint64)
        np.savez_compressed(OUT / "tfs_counters.npz", **c)

        # c1 from this repository's generator
        cfg = configs.make("c1")
        g1, w1 = tmp / "c1.gatbin", tmp / "c1.gatwgt"
        G.save_graph(cfg.graph, g1)
        G.save_model(cfg.model, w1)
        manifest["config1_gatbin_sha256"] = sha256(g1)
        manifest["config1_gatwgt_sha256"] = sha256(w1)
        d = tmp / "c1"
        d.mkdir()
        subprocess.run([str(DUMP), "chain", str(g1), str(w1), str(d)], check=True)
        np.savez_compressed(OUT / "config1.npz", **chain_npz(d, 1024, 40))

        # boundaries.cpp cases
        d = tmp / "bnd"
        d.mkdir()
        subprocess.run([str(DUMP), "boundary", str(d)], check=True)
        b = dict(perm=load(d, "bnd_perm.u32", np.uint32), steps=load(d, "bnd_steps.u64", np.uint64),
                 row=load(d, "bnd_row.u64", np.uint64), col=load(d, "bnd_col.u32", np.uint32))
        for D in (17, 33, 128, 256):
            for K in (1, 2, 4, 8):
                for dd in (7, 32, 40, 47):
                    key = f"{D}_{K}_{dd}"
                    b["ref_" + key] = load(d, f"bnd_{key}_ref.f32").reshape(35, K * dd)
                    if D in (17, 256) and K in (1, 8):
                        b["b0bf16_" + key] = load(d, f"bnd_{key}_b0bf16.f32").reshape(35, K * dd)
                    # Pins oracle_boundary_params to the reference's draws.
                    b["wsum_" + key] = np.array([load(d, f"bnd_{key}_w.f32").astype(np.float64).sum(),
                                                 load(d, f"bnd_{key}_al.f32").astype(np.float64).sum(),
                                                 load(d, f"bnd_{key}_ar.f32").astype(np.float64).sum()])
        np.savez_compressed(OUT / "boundary.npz", **b)

        # TFS family (ref_dump tfs), a subset of the boundary shapes
        d = tmp / "tfs"
        d.mkdir()
        subprocess.run([str(DUMP), "tfs", str(d)], check=True)
        t = {}
        for D, K, dd in TFS_CASES:
            key = f"{D}_{K}_{dd}"
            pre = f"tfs_{key}_"
            for name in ("lbf", "rbf", "l32", "r32", "max", "b1_den", "online16_den", "online16_max",
                         "block32_den", "block32_max", "hybrid32_den", "hybrid32_max"):
                t[f"{name}_{key}"] = load(d, pre + name + ".f32").reshape(35, K)
            t[f"blr_{key}"] = load(d, pre + "blr.f32").reshape(D, 2 * K)
            for name in ("b1_out", "online16_out", "block32_out", "hybrid32_out"):
                t[f"{name}_{key}"] = load(d, pre + name + ".f32").reshape(35, K * dd)
        np.savez_compressed(OUT / "tfs.npz", **t)

        # GATFIX1 fixture from the reference's export-fixture mode
        sg = small_fixture_graph()
        G.save_graph(sg, OUT / "fixture_small.gatbin")
        baseline = ROOT / "oracle" / "_ref" / "gat_baseline"
        subprocess.run([str(baseline), "--graph", str(OUT / "fixture_small.gatbin"), "--seed", "11", "--mode",
                        "export-fixture", "--layer", "1", "--fixture", str(OUT / "fixture_small_l1.gatfix"),
                        "--threads", "4"], check=True, stdout=subprocess.DEVNULL)
        manifest["fixture_small_gatbin_sha256"] = sha256(OUT / "fixture_small.gatbin")
        manifest["fixture_small_l1_gatfix_sha256"] = sha256(OUT / "fixture_small_l1.gatfix")
    (OUT / "MANIFEST.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
