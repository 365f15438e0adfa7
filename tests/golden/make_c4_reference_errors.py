"""Records the reference's own BF16 error on the headline configuration c4.

    python tests/golden/make_c4_reference_errors.py [--threads T]

Writes c4's GATBIN1 graph and GATWGT1 weights (this repository's seeded
generator), runs the reference's B0 driver built from its sources
(oracle/_ref/gat_baseline, bench/main.cpp benchmark mode with --output) once
on path standard_fp32 and once on standard_bf16, and stores in
tests/golden/c4_reference_errors.json the relative L2 and max-abs distance of
the reference's BF16 logits from its FP32 logits: the BF16 error floor of the
reference on the same bytes the GPU tests read. Run after
`make -C oracle ref`; takes a few minutes on 8 cores.
"""
import argparse
import hashlib
import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "gat-tfs_b200"))
import configs  # noqa: E402
import gatb200 as G  # noqa: E402

REF_BIN = ROOT / "oracle" / "_ref" / "gat_baseline"
OUT = Path(__file__).resolve().parent / "c4_reference_errors.json"


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 24), b""):
            h.update(b)
    return h.hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=8)
    args = ap.parse_args()
    cfg = configs.make("c4")
    with tempfile.TemporaryDirectory() as td:
        g, w = Path(td) / "c4.gatbin", Path(td) / "c4.gatwgt"
        G.save_graph(cfg.graph, g)
        G.save_model(cfg.model, w)
        out = {}
        for path in ("standard_fp32", "standard_bf16"):
            o = Path(td) / f"{path}.f32"
            subprocess.run([str(REF_BIN), "--graph", str(g), "--weights", str(w), "--path", path, "--mode",
                            "benchmark", "--threads", str(args.threads), "--warmups", "0", "--repeats", "1",
                            "--output", str(o)], check=True, capture_output=True)
            out[path] = np.fromfile(o, np.float32)
        a, b = out["standard_fp32"], out["standard_bf16"]
        rec = {
            "config": "c4", "nodes": cfg.graph.n, "edges": cfg.graph.e,
            "gatbin_sha256": sha256(g), "gatwgt_sha256": sha256(w),
            "reference_bf16_vs_fp32": {"relative_l2": float(np.linalg.norm(b - a) / np.linalg.norm(a)),
                                       "max_abs": float(np.abs(b - a).max()),
                                       "fp32_max_abs_value": float(np.abs(a).max())},
            "how": "oracle/_ref/gat_baseline --mode benchmark --warmups 0 --repeats 1 --output, paths "
                   "standard_fp32 and standard_bf16 (the reference's B0, bench/main.cpp:156-181)",
        }
    OUT.write_text(json.dumps(rec, indent=1) + "\n")
    print(json.dumps(rec))


if __name__ == "__main__":
    main()
