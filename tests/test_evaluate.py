"""Task evaluation of exported logits (gat-tfs_b200/evaluate.py), the
counterpart of the reference's evaluator and its tests
(baseline/scripts/evaluate_task.py, baseline/tests/evaluate_task_test.py):
perfect predictions, the accuracy-drop gate, and every input rejection. The GPU
case exports logits with the C++ driver (--output) for a BF16 and the FP32 path
and scores the BF16 run against the FP32 one (labels from the FP32 arg-max:
there are no real labels or checkpoints for the synthetic graphs)."""
import json
import struct
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
SCRIPT = ROOT / "gat-tfs_b200" / "evaluate.py"


def _run(tmp, actual: bytes, labels="0\n1\n0\n", split="0\n1\n2\n", gate=True, reference=True):
    (tmp / "actual.f32").write_bytes(actual)
    (tmp / "reference.f32").write_bytes(struct.pack("<6f", 2, 1, 3, 4, 7, 6))
    (tmp / "labels.csv").write_text(labels)
    (tmp / "split.csv").write_text(split)
    cmd = [sys.executable, str(SCRIPT), "--output", str(tmp / "actual.f32"), "--nodes", "3", "--classes", "2",
           "--labels", str(tmp / "labels.csv"), "--split", str(tmp / "split.csv")]
    if reference:
        cmd += ["--reference", str(tmp / "reference.f32")]
    if gate:
        cmd += ["--max-accuracy-drop", "0.05"]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=120)


GOOD = struct.pack("<6f", 2, 1, 3, 4, 7, 6)


def test_perfect_predictions(tmp_path):
    r = _run(tmp_path, GOOD)
    assert r.returncode == 0, r.stderr
    rep = json.loads(r.stdout)
    assert rep["accuracy"] == 1 and rep["gate"] == "PASS" and rep["prediction_agreement"] == 1
    assert rep["split_nodes"] == 3 and rep["accuracy_drop"] == 0


def test_accuracy_drop_gate_fails(tmp_path):
    r = _run(tmp_path, struct.pack("<6f", 1, 2, 3, 4, 7, 6))
    assert r.returncode == 1
    rep = json.loads(r.stdout)
    assert rep["gate"] == "FAIL" and abs(rep["accuracy_drop"] - 1 / 3) < 1e-12


def test_report_without_gate(tmp_path):
    r = _run(tmp_path, GOOD, gate=False, reference=False)
    assert r.returncode == 0
    assert json.loads(r.stdout) == {"accuracy": 1.0, "split_nodes": 3, "gate": "UNCONFIGURED"}


@pytest.mark.parametrize("case", ["nonfinite_logits", "wrong_logits_size", "duplicate_split", "out_of_range_split",
                                  "out_of_range_label", "fractional_label", "gate_without_reference"])
def test_invalid_inputs_rejected(tmp_path, case):
    kw = {}
    actual = GOOD
    if case == "nonfinite_logits":
        actual = struct.pack("<6f", float("nan"), 2, 3, 4, 7, 6)
    elif case == "wrong_logits_size":
        actual = GOOD[:-4]
    elif case == "duplicate_split":
        kw["split"] = "0\n0\n2\n"
    elif case == "out_of_range_split":
        kw["split"] = "0\n1\n3\n"
    elif case == "out_of_range_label":
        kw["labels"] = "0\n1\n2\n"
    elif case == "fractional_label":
        kw["labels"] = "0\n0.5\n1\n"
    elif case == "gate_without_reference":
        kw["reference"] = False
    r = _run(tmp_path, actual, **kw)
    assert r.returncode != 0 and "ValueError" in r.stderr, (case, r.stdout, r.stderr)


def test_npy_inputs_and_first_argmax(tmp_path):
    sys.path.insert(0, str(SCRIPT.parent))
    import evaluate as E
    logits = np.array([[1, 1, 0], [0, 2, 2], [5, 1, 5]], np.float32)  # ties: the first maximum wins
    logits.tofile(tmp_path / "l.f32")
    np.save(tmp_path / "lab.npy", np.array([0, 1, 0]))
    np.save(tmp_path / "sp.npy", np.array([2, 0, 1]))
    rep = E.evaluate(str(tmp_path / "l.f32"), 3, 3, np.load(tmp_path / "lab.npy"), np.load(tmp_path / "sp.npy"))
    assert rep["accuracy"] == 1.0


@pytest.mark.gpu
def test_driver_export_then_evaluate(tmp_path):
    """--output of the C++ driver on the small fixture graph, BF16 scored against FP32."""
    from test_cli import GOLDEN, run
    outs = {}
    for path in ("standard_fp32", "standard_bf16"):
        f = tmp_path / f"{path}.f32"
        r = run("--graph", str(GOLDEN / "fixture_small.gatbin"), "--seed", "11", "--path", path, "--mode",
                "benchmark", "--repeats", "1", "--warmups", "1", "--output", str(f))
        assert r.returncode == 0, r.stderr
        outs[path] = f
    ref = np.fromfile(outs["standard_fp32"], "<f4")
    nodes = 200
    classes = ref.size // nodes
    assert ref.size == nodes * classes
    labels = ref.reshape(nodes, classes).argmax(1)
    np.save(tmp_path / "labels.npy", labels)
    np.save(tmp_path / "split.npy", np.arange(0, nodes, 2))
    r = subprocess.run([sys.executable, str(SCRIPT), "--output", str(outs["standard_bf16"]), "--nodes", str(nodes),
                        "--classes", str(classes), "--labels", str(tmp_path / "labels.npy"), "--split",
                        str(tmp_path / "split.npy"), "--reference", str(outs["standard_fp32"]),
                        "--max-accuracy-drop", "0.05"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    rep = json.loads(r.stdout)
    assert rep["gate"] == "PASS" and rep["reference_accuracy"] == 1.0 and rep["prediction_agreement"] >= 0.95
