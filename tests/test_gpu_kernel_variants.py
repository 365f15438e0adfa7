"""The aggregation kernel variants that are not the default for their shape,
selected per process by environment variable (GAT_B200_NARROW_AGG=pair: the
lane-pair kernel for narrow single-head layers; GAT_B200_NARROW_AGG=gather4:
single-head rows fetched by the TMA row gather, here 40 columns = 5 vectors
per row; GAT_B200_HIDDEN_AGG=gather4: hidden-layer rows fetched by the TMA row
gather), each in a child process on
the c2 graph (hubs split into segments, wide rows, short rows): the
three-layer BF16 forward against the R0 oracle (relative L2 <= 1e-2) and
against the default kernels' forward (relative L2 <= 2e-3: the same math in
another summation order)."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

CHILD = r"""
import sys, numpy as np, torch
sys.path[:0] = [{pkg!r}, {orc!r}]
import configs, gatb200 as G, oracle as O
cfg = configs.make("c2")
g = G.DeviceGraph(cfg.graph.row, cfg.graph.col)
m = G.DeviceModel(g, [G.DeviceLayer(p) for p in cfg.model], G.PATH_STANDARD_BF16)
y = torch.empty((cfg.graph.n, m.classes), dtype=torch.float32, device="cuda")
m.forward(torch.from_numpy(cfg.graph.x).cuda(), y, False, False)
torch.cuda.synchronize(); G.check_device()
np.save({out!r}, y.cpu().numpy())
"""


def _forward(tmp_path, name, env_extra):
    out = tmp_path / f"{name}.npy"
    code = CHILD.format(pkg=str(ROOT / "gat-tfs_b200"), orc=str(ROOT / "oracle"), out=str(out))
    env = dict(os.environ, **env_extra)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    return np.load(out)


@pytest.fixture(scope="module")
def reference_logits():
    import configs
    import oracle as O
    cfg = configs.make("c2")
    model = [(p.w, p.al, p.ar, p.heads, p.dim) for p in cfg.model]
    return O.ref_chain(cfg.graph.row, cfg.graph.col, cfg.graph.x, model)[2]["out"]


@pytest.mark.parametrize("name,env", [("default", {}), ("narrow_pair", {"GAT_B200_NARROW_AGG": "pair"}),
                                      ("narrow_gather4", {"GAT_B200_NARROW_AGG": "gather4"}),
                                      ("hidden_gather4", {"GAT_B200_HIDDEN_AGG": "gather4"})])
def test_variant_forward(tmp_path, reference_logits, name, env):
    got = _forward(tmp_path, name, env)
    ref = reference_logits
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert np.isfinite(got).all() and rel <= 1e-2, (name, rel)
    if name != "default":
        base = _forward(tmp_path, "default_" + name, {})
        d = np.linalg.norm(got - base) / np.linalg.norm(base)
        assert d <= 2e-3, (name, d)
