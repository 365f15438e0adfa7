"""ctypes wrapper of oracle/_build/libgat_oracle.so (the CPU checker).

TEST INFRASTRUCTURE: only tests/, __graft_entry__.smoke() and bench.py's CPU
legs import this module, and only to check or time against it. The product
path (gat-tfs_b200/libgat_b200.so and gatb200.py) never does.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libgat_oracle.so"


def build():
    subprocess.run(["make", "-s", "-C", str(HERE), "all"], check=True)


if not LIB.exists():
    build()
_lib = C.CDLL(str(LIB))

_u64p = C.POINTER(C.c_uint64)
_u32p = C.POINTER(C.c_uint32)
_f32p = C.POINTER(C.c_float)
_u16p = C.POINTER(C.c_uint16)

_lib.oracle_rne.restype = C.c_uint16
_lib.oracle_rne.argtypes = [C.c_float]
_lib.oracle_degree_schedule.restype = C.c_uint64
_lib.oracle_degree_schedule.argtypes = [C.c_uint64, _u64p, _u32p]
_layer_args = [C.c_uint64, _u64p, _u32p, C.c_int, C.c_int, C.c_int, _f32p, _f32p, _f32p, _f32p, C.c_int]
_lib.oracle_ref_layer.argtypes = _layer_args + [_f32p] * 7
_lib.oracle_fp64_layer.argtypes = [C.c_uint64, _u64p, _u32p, C.c_int, C.c_int, C.c_int, _f32p, _f32p, _f32p, _f32p, _f32p]
_lib.oracle_b0_layer.argtypes = _layer_args + [C.c_int, C.c_int] + [_f32p] * 6
_lib.oracle_max_prescan.argtypes = [C.c_uint64, _u64p, _u32p, C.c_int, _f32p, _f32p, _f32p]
_lib.oracle_standard_aggregate.argtypes = [C.c_uint64, _u64p, _u32p, C.c_int, C.c_int] + [_f32p] * 8
_lib.oracle_finish.argtypes = [C.c_uint64, C.c_int, C.c_int, _f32p, C.c_int, _f32p]
_lib.oracle_tfs_aggregate.argtypes = ([C.c_uint64, _u64p, _u32p, C.c_int, C.c_int, C.c_int] + [_f32p] * 7 +
                                      [C.c_int, C.c_int, C.c_int] + [_f32p] * 3)
_lib.oracle_prepare_blr.argtypes = [C.c_int, C.c_int, C.c_int, _f32p, _f32p, _f32p, _f32p]
_lib.oracle_lr_reordered.argtypes = [C.c_uint64, C.c_int, C.c_int, _f32p, _f32p, _f32p, C.c_int, _f32p, _f32p]
_lib.oracle_boundary_params.argtypes = [C.c_int, C.c_int, C.c_int, _f32p, _f32p, _f32p]
_lib.oracle_random_layer.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, _f32p, _f32p, _f32p]


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


def _f(a):
    return np.ascontiguousarray(a, np.float32)


def rne(x: float) -> int:
    return _lib.oracle_rne(x)


def quantize(a: np.ndarray) -> np.ndarray:
    """FP32 -> BF16 RNE -> FP32 (common.cpp:94-96)."""
    u = _f(a).view(np.uint32).astype(np.uint64)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x7FFFFF) != 0)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = np.where(nan, (u >> 16) | 0x40, r)
    return (r.astype(np.uint32) << 16).view(np.float32)


def degree_schedule(row: np.ndarray):
    row = np.ascontiguousarray(row, np.uint64)
    n = len(row) - 1
    perm = np.empty(n, np.uint32)
    steps = _lib.oracle_degree_schedule(n, _p(row, _u64p), _p(perm, _u32p))
    return perm, int(steps)


def ref_layer(row, col, x, w, al, ar, heads, dim, hidden, want_p=False):
    """R0 (ref_fp32.cpp:3-26). Returns dict of out/z/left/right/max/den(/p)."""
    row = np.ascontiguousarray(row, np.uint64)
    col = np.ascontiguousarray(col, np.uint32)
    x, w, al, ar = _f(x), _f(w), _f(al), _f(ar)
    n, e, width = len(row) - 1, len(col), heads * dim
    o = {k: np.empty((n, heads), np.float32) for k in ("left", "right", "max", "den")}
    o["z"] = np.empty((n, width), np.float32)
    o["out"] = np.empty((n, width), np.float32)
    p = np.empty((e, heads), np.float32) if want_p else None
    _lib.oracle_ref_layer(n, _p(row, _u64p), _p(col, _u32p), x.shape[1], heads, dim, _p(x, _f32p), _p(w, _f32p),
                          _p(al, _f32p), _p(ar, _f32p), int(hidden), _p(o["z"], _f32p), _p(o["left"], _f32p),
                          _p(o["right"], _f32p), _p(o["max"], _f32p), _p(o["den"], _f32p), _p(p, _f32p),
                          _p(o["out"], _f32p))
    if want_p:
        o["p"] = p
    return o


def fp64_layer(row, col, x, w, al, ar, heads, dim):
    """boundaries.cpp:15-21 FP64 oracle (no activation)."""
    row = np.ascontiguousarray(row, np.uint64)
    col = np.ascontiguousarray(col, np.uint32)
    x, w, al, ar = _f(x), _f(w), _f(al), _f(ar)
    n = len(row) - 1
    out = np.empty((n, heads * dim), np.float32)
    _lib.oracle_fp64_layer(n, _p(row, _u64p), _p(col, _u32p), x.shape[1], heads, dim, _p(x, _f32p), _p(w, _f32p),
                           _p(al, _f32p), _p(ar, _f32p), _p(out, _f32p))
    return out


def b0_layer(row, col, x, w, al, ar, heads, dim, hidden, bf16=True, round_z=False):
    """B0 standard_layer (baseline_standard.cpp:98-108); round_z emulates BF16 H storage."""
    row = np.ascontiguousarray(row, np.uint64)
    col = np.ascontiguousarray(col, np.uint32)
    x, w, al, ar = _f(x), _f(w), _f(al), _f(ar)
    n, width = len(row) - 1, heads * dim
    o = {k: np.empty((n, heads), np.float32) for k in ("left", "right", "max", "den")}
    o["z"] = np.empty((n, width), np.float32)
    o["out"] = np.empty((n, width), np.float32)
    _lib.oracle_b0_layer(n, _p(row, _u64p), _p(col, _u32p), x.shape[1], heads, dim, _p(x, _f32p), _p(w, _f32p),
                         _p(al, _f32p), _p(ar, _f32p), int(hidden), int(bf16), int(round_z), _p(o["z"], _f32p),
                         _p(o["left"], _f32p), _p(o["right"], _f32p), _p(o["max"], _f32p), _p(o["den"], _f32p),
                         _p(o["out"], _f32p))
    return o


_lib.oracle_online_counters.restype = None
_lib.oracle_online_counters.argtypes = [C.c_uint64, _u64p, _u32p, _u32p, C.c_int, _f32p, _f32p, C.c_int, _u64p,
                                        _u64p, _u64p, _u64p]


def online_counters(row, col, perm, left, right, heads, block):
    """icpp_online's exact counters (icpp_online.hpp:18-22): per (row, head)
    blocks / max updates / rescales [n][heads] and the totals
    (blocks, max_updates, rescales, rescale_events, neighbor_steps)."""
    row = np.ascontiguousarray(row, np.uint64)
    col = np.ascontiguousarray(col, np.uint32)
    perm = np.ascontiguousarray(perm, np.uint32)
    n = len(row) - 1
    rb, ru, rr = (np.zeros((n, heads), np.uint64) for _ in range(3))
    tot = np.zeros(5, np.uint64)
    _lib.oracle_online_counters(n, _p(row, _u64p), _p(col, _u32p), _p(perm, _u32p), heads, _p(_f(left), _f32p),
                                _p(_f(right), _f32p), block, _p(rb, _u64p), _p(ru, _u64p), _p(rr, _u64p),
                                _p(tot, _u64p))
    return rb, ru, rr, tot


def max_prescan(row, col, left, right, heads):
    row = np.ascontiguousarray(row, np.uint64)
    col = np.ascontiguousarray(col, np.uint32)
    n = len(row) - 1
    m = np.empty((n, heads), np.float32)
    _lib.oracle_max_prescan(n, _p(row, _u64p), _p(col, _u32p), heads, _p(_f(left), _f32p), _p(_f(right), _f32p),
                            _p(m, _f32p))
    return m


def standard_aggregate(row, col, z, left, right, mx, heads, dim, fixed_p=None, fixed_den=None):
    row = np.ascontiguousarray(row, np.uint64)
    col = np.ascontiguousarray(col, np.uint32)
    n = len(row) - 1
    out = np.empty((n, heads * dim), np.float32)
    den = np.empty((n, heads), np.float32)
    fp = None if fixed_p is None else _f(fixed_p)
    fd = None if fixed_den is None else _f(fixed_den)
    _lib.oracle_standard_aggregate(n, _p(row, _u64p), _p(col, _u32p), heads, dim, _p(_f(z), _f32p),
                                   _p(None if left is None else _f(left), _f32p),
                                   _p(None if right is None else _f(right), _f32p),
                                   _p(None if mx is None else _f(mx), _f32p), _p(fp, _f32p), _p(fd, _f32p),
                                   _p(out, _f32p), _p(den, _f32p))
    return out, den


def finish(out, den, heads, dim, hidden):
    out = _f(out).copy()
    n = out.shape[0]
    _lib.oracle_finish(n, heads, dim, _p(_f(den), _f32p), int(hidden), _p(out, _f32p))
    return out


TFS_EDGE, TFS_BLOCK, TFS_SPLIT = 0, 1, 2


def tfs_aggregate(row, col, xq, wq, left, right, heads, dim, mx=None, rounding=TFS_EDGE, block=0, threshold=1,
                  fixed_p=None, fixed_den=None):
    """TFS aggregation family (baseline_tfs.cpp:16-110, icpp_online/icpp_block/
    icpp_heads_hybrid; see gat_oracle.h). xq, wq: BF16-valued FP32 arrays.
    Returns (unnormalized out [n][heads*dim], den [n][heads], max [n][heads])."""
    row = np.ascontiguousarray(row, np.uint64)
    col = np.ascontiguousarray(col, np.uint32)
    xq, wq = _f(xq), _f(wq)
    n = len(row) - 1
    out = np.empty((n, heads * dim), np.float32)
    den = np.empty((n, heads), np.float32)
    mo = np.empty((n, heads), np.float32)
    _lib.oracle_tfs_aggregate(n, _p(row, _u64p), _p(col, _u32p), xq.shape[1], heads, dim, _p(xq, _f32p),
                              _p(wq, _f32p), _p(None if left is None else _f(left), _f32p),
                              _p(None if right is None else _f(right), _f32p),
                              _p(None if mx is None else _f(mx), _f32p),
                              _p(None if fixed_p is None else _f(fixed_p), _f32p),
                              _p(None if fixed_den is None else _f(fixed_den), _f32p), int(rounding), int(block),
                              int(threshold), _p(out, _f32p), _p(den, _f32p), _p(mo, _f32p))
    return out, den, mo


def prepare_blr(w, al, ar, heads, dim):
    """common.cpp:100-106: blr [in][2*heads] (L columns, then R columns)."""
    w = _f(w)
    blr = np.empty((w.shape[0], 2 * heads), np.float32)
    _lib.oracle_prepare_blr(w.shape[0], heads, dim, _p(w, _f32p), _p(_f(al), _f32p), _p(_f(ar), _f32p),
                            _p(blr, _f32p))
    return blr


def lr_reordered(x, blr, heads, policy):
    """baseline_standard.cpp:29-43; policy 0 = "bf16" (BF16 X, RNE(blr)), 1 = "fp32"."""
    x = _f(x)
    xq = quantize(x)
    n = x.shape[0]
    left = np.empty((n, heads), np.float32)
    right = np.empty((n, heads), np.float32)
    _lib.oracle_lr_reordered(n, x.shape[1], heads, _p(x, _f32p), _p(xq, _f32p), _p(_f(blr), _f32p), int(policy),
                             _p(left, _f32p), _p(right, _f32p))
    return left, right


def tfs_layer(row, col, x, w, al, ar, heads, dim, hidden, policy=0, rounding=TFS_EDGE, block=0, threshold=1):
    """baseline_tfs.cpp:111-117 (tfs_layer): convert, lr_reordered, max_prescan,
    tfs_aggregate, finish. rounding/block/threshold select the icpp_* variants
    (their layer() functions run the same stages, icpp_block.cpp:329-352)."""
    xq = quantize(x)
    blr = prepare_blr(w, al, ar, heads, dim)
    left, right = lr_reordered(x, blr, heads, policy)
    mx = max_prescan(row, col, left, right, heads) if rounding == TFS_EDGE and block == 0 else None
    out, den, _ = tfs_aggregate(row, col, xq, quantize(w), left, right, heads, dim, mx=mx, rounding=rounding,
                                block=block, threshold=threshold)
    return finish(out, den, heads, dim, hidden)


def boundary_params(D, K, d):
    w = np.empty((D, K * d), np.float32)
    al = np.empty(K * d, np.float32)
    ar = np.empty(K * d, np.float32)
    _lib.oracle_boundary_params(D, K, d, _p(w, _f32p), _p(al, _f32p), _p(ar, _f32p))
    return w, al, ar


def boundary_graph(D):
    """boundaries.cpp:10-13: 35 nodes, degrees cycling {0,1,2,15,16,17,31,32,33,63,64,65,129}."""
    deg = [0, 1, 2, 15, 16, 17, 31, 32, 33, 63, 64, 65, 129]
    row, col = [0], []
    for i in range(35):
        for e in range(deg[i % 13]):
            col.append((i * 3 + e * 7) % 35)
        row.append(len(col))
    x = (np.sin(np.arange(35 * D, dtype=np.float32) * np.float32(0.17)) * np.float32(0.5)).astype(np.float32)
    return np.array(row, np.uint64), np.array(col, np.uint32), x.reshape(35, D)


def random_model(din, classes, seed):
    m = []
    for l, (i, h, d) in enumerate([(din, 8, 32), (256, 8, 32), (256, 1, classes)]):
        w = np.empty((i, h * d), np.float32)
        al = np.empty(h * d, np.float32)
        ar = np.empty(h * d, np.float32)
        _lib.oracle_random_layer(l, din, classes, seed, _p(w, _f32p), _p(al, _f32p), _p(ar, _f32p))
        m.append((w, al, ar, h, d))
    return m


def ref_chain(row, col, x, model):
    """Three R0 layers, hidden ELU in layers 1-2 (bench/main.cpp:93-94)."""
    outs = []
    inp = x
    for l, (w, al, ar, h, d) in enumerate(model):
        o = ref_layer(row, col, inp, w, al, ar, h, d, l < 2)
        outs.append(o)
        inp = o["out"]
    return outs


def errors(ref: np.ndarray, got: np.ndarray) -> dict:
    """The reference's error metrics (common.cpp:141-150)."""
    ref = np.asarray(ref, np.float64).ravel()
    got = np.asarray(got, np.float64).ravel()
    if ref.size == 0 or ref.size != got.size:
        raise ValueError("comparison size mismatch")
    fin = np.isfinite(ref) & np.isfinite(got)
    if not fin.all():
        return dict(finite=False, max_abs=np.inf, relative_l2=np.inf)
    d = got - ref
    den = float(np.dot(ref, ref))
    sq = float(np.dot(d, d))
    return dict(finite=True, max_abs=float(np.abs(d).max()), mean_abs=float(np.abs(d).mean()),
                relative_l2=(np.sqrt(sq / den) if den > 0 else (0.0 if sq == 0 else np.inf)),
                rmse=float(np.sqrt(sq / ref.size)))
