"""The online TFS variants of the C++ mirror (include/gat_b200.hpp):
icpp_online, icpp_block and icpp_heads_hybrid with the reference's signatures
(baseline/tfs_online/icpp_online.hpp:37-43, icpp_block.hpp:33-39,
icpp_heads_hybrid.hpp:18-24), through tests/cpp/mirror_test.cpp --gpu-online:
every layer against the FP64 layer at the TFS gate, the exact counters against
what the CSR and the degree schedule determine, aggregate() + finish against
layer(), and heads_hybrid's fallback to icpp_block outside heads 8, dim 32.
The kernels underneath are checked against the oracle in test_gpu_tfs.py; this
file is collected late so that a failure here leaves those already run, and it
also passes when run on its own.
"""
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "gat-tfs_b200"

pytestmark = pytest.mark.gpu


def test_online_variants(tmp_path):
    exe = tmp_path / "mirror_test"
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-Wextra", "-I", str(ROOT / "include"),
           str(ROOT / "tests" / "cpp" / "mirror_test.cpp"), "-L", str(PKG), "-lgat_b200",
           f"-Wl,-rpath,{PKG}", "-o", str(exe)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe), "--gpu-online", str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "MIRROR PASS online cases=16" in r.stdout
