"""Node-classification evaluation of exported logits (outside any timing).

Counterpart of the reference's task evaluator (baseline/scripts/evaluate_task.py):
same command line, same input rules and the same JSON report, so a run that
exported its logits with the driver's --output (FP32 row-major [nodes][classes],
little endian) is scored the same way.

  python evaluate.py --output LOGITS --nodes N --classes C --labels L --split S
                     [--reference REF_LOGITS [--max-accuracy-drop X]]

labels: one integer class per node; split: the node ids to score (not a mask);
both as .npy or as comma/newline separated text (.csv, .csv.gz). Prediction =
first arg-max of a node's logits. With --reference the report adds the
reference's accuracy, the accuracy drop and the prediction agreement; with
--max-accuracy-drop it also carries gate PASS/FAIL and the exit status is 1 on
FAIL. Invalid inputs raise ValueError (exit status 1).
"""
from __future__ import annotations

import argparse
import json
import sys
from typing import Optional, Sequence

import numpy as np


def _read_array(path: str) -> np.ndarray:
    if path.endswith(".npy"):
        return np.load(path, allow_pickle=False)
    return np.loadtxt(path, delimiter=",")


def read_logits(path: str, nodes: int, classes: int) -> np.ndarray:
    v = np.fromfile(path, dtype="<f4")
    if v.size != nodes * classes or not np.all(np.isfinite(v)):
        raise ValueError("invalid/nonfinite logits")
    return v.reshape(nodes, classes)


def _integers(a: np.ndarray) -> np.ndarray:
    if np.any(a != np.trunc(a)):
        raise ValueError("labels/split must be integers")
    return a.astype(np.int64)


def evaluate(output: str, nodes: int, classes: int, labels: np.ndarray, split: np.ndarray,
             reference: Optional[str] = None, max_accuracy_drop: Optional[float] = None) -> dict:
    """The report dict (and whether the gate passed, under key 'gate')."""
    labels = np.asarray(labels).reshape(-1)
    split = np.asarray(split).reshape(-1)
    if labels.size != nodes or not np.all(np.isfinite(labels)) or not np.all(np.isfinite(split)):
        raise ValueError("invalid label/split sizes or finite values")
    labels = _integers(labels)
    split = _integers(split)
    if split.size == 0 or split.min() < 0 or split.max() >= nodes or np.unique(split).size != split.size:
        raise ValueError("invalid or duplicate split IDs")
    want = labels[split]
    if want.min() < 0 or want.max() >= classes:
        raise ValueError("split labels out of bounds")
    pred = read_logits(output, nodes, classes)[split].argmax(axis=1)
    rep = {"accuracy": float(np.mean(pred == want)), "split_nodes": int(split.size), "gate": "UNCONFIGURED"}
    if reference:
        ref = read_logits(reference, nodes, classes)[split].argmax(axis=1)
        ref_acc = float(np.mean(ref == want))
        rep.update(reference_accuracy=ref_acc, accuracy_drop=ref_acc - rep["accuracy"],
                   prediction_agreement=float(np.mean(pred == ref)))
    if max_accuracy_drop is not None:
        if not reference or not np.isfinite(max_accuracy_drop) or max_accuracy_drop < 0:
            raise ValueError("accuracy drop gate needs reference and a finite nonnegative threshold")
        rep["gate"] = "PASS" if rep["accuracy_drop"] <= max_accuracy_drop else "FAIL"
    return rep


def main(argv: Optional[Sequence[str]] = None) -> int:
    ap = argparse.ArgumentParser(description="node classification accuracy of exported FP32 logits")
    ap.add_argument("--output", required=True, help="FP32 row-major model logits")
    ap.add_argument("--nodes", type=int, required=True)
    ap.add_argument("--classes", type=int, required=True)
    ap.add_argument("--labels", required=True)
    ap.add_argument("--split", required=True, help="development/test node IDs, not a boolean mask")
    ap.add_argument("--reference", help="FP32 R0 logits for accuracy-drop gate")
    ap.add_argument("--max-accuracy-drop", type=float)
    a = ap.parse_args(argv)
    rep = evaluate(a.output, a.nodes, a.classes, _read_array(a.labels), _read_array(a.split), a.reference,
                   a.max_accuracy_drop)
    print(json.dumps(rep))
    return 1 if rep["gate"] == "FAIL" else 0


if __name__ == "__main__":
    sys.exit(main())
