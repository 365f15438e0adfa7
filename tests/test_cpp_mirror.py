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


def test_mirror_host_checks(mirror_bin, tmp_path):
    r = subprocess.run([str(mirror_bin), "--host", str(tmp_path)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "MIRROR PASS host" in r.stdout and r.stdout.count("MIRROR PASS rejects") == 19


@pytest.mark.gpu
def test_mirror_layer_functions_on_gpu(mirror_bin, tmp_path):
    r = subprocess.run([str(mirror_bin), "--gpu", str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "MIRROR PASS gpu cases=12" in r.stdout
