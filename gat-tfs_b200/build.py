"""Builds libgat_b200.so in-tree (sm_100a only).

    python gat-tfs_b200/build.py [--verbose]

Each source compiles to an object under gat-tfs_b200/_build/ (in parallel), and
the objects link into gat-tfs_b200/libgat_b200.so with the CUDA runtime linked
statically, so the library needs only the NVIDIA driver at run time. The C++
drivers in cli/ (gat_b200_bench, gat_b200_tfs_online, gat_b200_tfs_adaptive) link against it. A source
is recompiled only when it or a header is newer than its object.
gat_b200_make_inputs links the host objects only (no CUDA runtime, no
libgat_b200.so).
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "_build"
LIB = PKG / "libgat_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fopenmp,-Wall",
                     "-I" + str(ROOT / "include"), "-Xptxas", "-v"]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-fopenmp", "-Wall", "-I" + str(ROOT / "include"),
             "-I/usr/local/cuda/include"]

# cli programs that need no GPU and must not load the library: the input
# writer of the CPU reference arm (bench.py --impl reference)
HOST_ONLY = {"gat_b200_make_inputs"}

# refrng.cpp must round like the reference's sources as oracle/Makefile builds
# them (g++ -O3 -mfma): std::normal_distribution is inline and contracts to FMA.
PER_FILE_FLAGS = {"refrng.cpp": ["-mfma"]}


def _headers():
    return list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h")) + list((ROOT / "include").glob("*.hpp"))


def _stale(src: Path, obj: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in _headers())


def _compile(src: Path, verbose: bool):
    obj = OUT / (src.stem + ".o")
    if not _stale(src, obj):
        return obj, ""
    if src.suffix == ".cu":
        cmd = [NVCC] + CUDA_FLAGS + ["-c", str(src), "-o", str(obj)]
    else:
        extra = PER_FILE_FLAGS.get(src.name, [])
        cmd = ["g++"] + CXX_FLAGS + extra + ["-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log = r.stdout + r.stderr
    (OUT / (src.stem + ".log")).write_text(log)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src.name}\n{log}")
    if verbose:
        print(log)
    return obj, log


def build(verbose: bool = False) -> Path:
    OUT.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = [f.result()[0] for f in [ex.submit(_compile, s, verbose) for s in sources]]
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-Xcompiler", "-fopenmp", "-o", str(LIB)] + [str(o) for o in objs] + ["-lgomp"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed\n" + r.stdout + r.stderr)
    # the C++ drivers over the C ABI (cli/*.cpp -> gat-tfs_b200/<name>): the
    # reference's bench/main.cpp and tfs_online/main.cpp interfaces
    hdr = max(h.stat().st_mtime for h in list((ROOT / "include").glob("*.h*")) + list((PKG / "cli").glob("*.hpp")))
    host_objs = [OUT / "host.o", OUT / "synth.o", OUT / "refrng.o"]
    for src in sorted((PKG / "cli").glob("*.cpp")):
        exe = PKG / src.stem
        if not exe.exists() or exe.stat().st_mtime < max(LIB.stat().st_mtime, src.stat().st_mtime, hdr):
            if src.stem in HOST_ONLY:
                # linked from the host objects alone: no CUDA, no libgat_b200.so
                cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-I" + str(ROOT / "include"), str(src)] + \
                      [str(o) for o in host_objs] + ["-fopenmp", "-o", str(exe)]
            else:
                cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-I" + str(ROOT / "include"), str(src), "-o", str(exe),
                       "-L" + str(PKG), "-lgat_b200", "-Wl,-rpath,$ORIGIN"]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"driver build failed: {src.name}\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(args.verbose))
    sys.exit(0)
