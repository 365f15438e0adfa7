"""Python host mirror of the reference's GAT API over libgat_b200.so (ctypes).

The reference's C++ surface (baseline/include/gat.hpp) is mirrored by name:
Graph / Param / Model, load_graph / save_graph, load_model / save_model,
random_model, degree_schedule, projection, max_prescan, standard_aggregate,
finish, standard_layer, plus the fused layer and the three-layer model that
the benchmark runs. Errors raise GatError (the reference raises
std::runtime_error with the same messages).

Device buffers are torch CUDA tensors; torch is only used for device memory,
streams and the process group, never for the computation. The library is the
in-tree build gat-tfs_b200/libgat_b200.so; importing this module fails if it is
missing (there is no fallback path).
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass, field
from pathlib import Path
from typing import List, Optional, Sequence

import numpy as np

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("GAT_B200_LIB", _PKG / "libgat_b200.so"))
if not LIB_PATH.exists():
    raise ImportError(f"{LIB_PATH} is missing: build it with `python gat-tfs_b200/build.py`")
_lib = C.CDLL(str(LIB_PATH))

F32, BF16 = 0, 1
PATH_STANDARD_BF16, PATH_STANDARD_FP32, PATH_TFS_BF16, PATH_ADAPTIVE_BF16, PATH_MATCHED_ATTENTION = 0, 1, 2, 3, 4
TFS_EDGE, TFS_BLOCK, TFS_SPLIT = 0, 1, 2
LR_BF16, LR_FP32 = 0, 1
PATHS = {"standard_bf16": PATH_STANDARD_BF16, "standard_fp32": PATH_STANDARD_FP32}
OK, EINVAL, ECUDA, EUNSUPPORTED, ETIMEOUT, EIO = range(6)

_u64p = C.POINTER(C.c_uint64)
_u32p = C.POINTER(C.c_uint32)
_u16p = C.POINTER(C.c_uint16)
_f32p = C.POINTER(C.c_float)
_vp = C.c_void_p

# (name, restype, argtypes) of every exported entry point, as declared in
# include/gat_b200.h.
SIGNATURES = [
    ("gat_b200_last_error", C.c_char_p, []),
    ("gat_b200_version", C.c_int, []),
    ("gat_b200_padded_ld", C.c_int, [C.c_int, C.c_int]),
    ("gat_b200_rne", C.c_uint16, [C.c_float]),
    ("gat_b200_convert_host", C.c_int, [_f32p, _u16p, C.c_uint64]),
    ("gat_b200_validate_csr", C.c_int, [C.c_uint64, C.c_uint64, _u64p, _u32p]),
    ("gat_b200_read_graph_header", C.c_int, [C.c_char_p, _u64p, _u64p, _u32p, _u32p]),
    ("gat_b200_read_graph", C.c_int, [C.c_char_p, C.c_uint64, C.c_uint64, C.c_uint32, _u64p, _u32p, _f32p]),
    ("gat_b200_write_graph", C.c_int, [C.c_char_p, C.c_uint64, C.c_uint64, C.c_uint32, C.c_uint32, _u64p, _u32p, _f32p]),
    ("gat_b200_read_weights", C.c_int, [C.c_char_p, C.c_int, C.c_int, C.POINTER(_f32p), C.POINTER(_f32p), C.POINTER(_f32p)]),
    ("gat_b200_write_weights", C.c_int, [C.c_char_p, C.c_int, C.c_int, C.POINTER(_f32p), C.POINTER(_f32p), C.POINTER(_f32p)]),
    ("gat_b200_write_fixture", C.c_int, [C.c_char_p, C.c_uint64, C.c_uint64, C.c_int, C.c_int, C.c_int, _u64p, _u32p,
                                         _f32p, _f32p, _f32p, _f32p, _f32p, _f32p]),
    ("gat_b200_read_fixture", C.c_int, [C.c_char_p, C.c_uint64, C.c_uint64, C.c_int, C.c_int, C.c_int, _u64p, _u32p,
                                        _f32p, _f32p, _f32p, _f32p, _f32p, _f32p]),
    ("gat_b200_random_model", C.c_int, [C.c_int, C.c_int, C.c_int, C.POINTER(_f32p), C.POINTER(_f32p), C.POINTER(_f32p)]),
    ("gat_b200_synth_uniform_graph", C.c_int, [C.c_uint64, C.c_uint32, C.c_uint64, _u64p, _u32p]),
    ("gat_b200_synth_powerlaw_graph", C.c_int, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_double, C.c_uint64, _u64p, _u32p]),
    ("gat_b200_synth_normal", C.c_int, [C.c_uint64, C.c_double, C.c_uint64, C.c_uint64, _f32p]),
    ("gat_b200_synth_normal_range", C.c_int, [C.c_uint64, C.c_uint64, C.c_double, C.c_uint64, C.c_uint64, _f32p]),
    ("gat_b200_synth_powerlaw_rows", C.c_int, [C.c_uint64, C.c_uint64, C.c_uint64, C.c_double, C.c_uint64, C.c_uint64, C.c_uint64, _u64p, _u32p]),
    ("gat_b200_synth_uniform", C.c_int, [C.c_uint64, C.c_double, C.c_double, C.c_uint64, C.c_uint64, _f32p]),
    ("gat_b200_synth_rmat", C.c_int, [C.c_int, C.c_uint64, C.c_double, C.c_double, C.c_double, C.c_uint64,
                                      C.c_uint64, C.c_uint64, _u64p, _u32p, _u64p]),
    ("gat_b200_graph_create", C.c_int, [C.c_uint64, C.c_uint64, _u64p, _u32p, _vp, C.POINTER(_vp)]),
    ("gat_b200_graph_create_part", C.c_int, [C.c_uint64, C.c_uint64, C.c_uint64, _u64p, _u32p, _vp, C.POINTER(_vp)]),
    ("gat_b200_graph_destroy", C.c_int, [_vp]),
    ("gat_b200_graph_schedule", C.c_int, [_vp, _u32p, _u64p]),
    ("gat_b200_graph_device_csr", C.c_int, [_vp, C.POINTER(_vp), C.POINTER(_vp)]),
    ("gat_b200_graph_info", C.c_int, [_vp, _u64p, _u64p, _u32p, _u32p, _u32p, _u32p]),
    ("gat_b200_layer_create", C.c_int, [C.c_int, C.c_int, C.c_int, _f32p, _f32p, _f32p, C.POINTER(_vp)]),
    ("gat_b200_layer_destroy", C.c_int, [_vp]),
    ("gat_b200_convert", C.c_int, [C.c_uint64, C.c_int, _vp, C.c_int, _vp, C.c_int, _vp]),
    ("gat_b200_projection", C.c_int, [_vp, C.c_uint64, _vp, C.c_int, C.c_int, _vp, C.c_int, C.c_int, _vp, _vp, _vp]),
    ("gat_b200_max_prescan", C.c_int, [_vp, C.c_int, _vp, _vp, _vp, _vp]),
    ("gat_b200_edge_softmax", C.c_int, [_vp, C.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("gat_b200_standard_aggregate", C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp, C.c_int, _vp, _vp, _vp]),
    ("gat_b200_finish", C.c_int, [C.c_uint64, C.c_int, C.c_int, _vp, C.c_int, _vp, C.c_int, _vp]),
    ("gat_b200_aggregate_fused", C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_int, C.c_int, _vp, _vp, C.c_int, _vp, C.c_int, C.c_int, _vp]),
    ("gat_b200_aggregate_fused_noalloc", C.c_int, [C.c_uint64, C.c_uint64, _vp, _vp, C.c_int, C.c_int, _vp, C.c_int, C.c_int, _vp, _vp, C.c_int, _vp, C.c_int, C.c_int, _vp]),
    ("gat_b200_standard_layer", C.c_int, [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp, _vp, C.c_int, C.c_int, _vp]),
    ("gat_b200_lr_reordered", C.c_int, [_vp, C.c_uint64, _vp, C.c_int, C.c_int, C.c_int, _vp, C.c_int, _vp, _vp, _vp]),
    ("gat_b200_tfs_aggregate", C.c_int, [_vp, _vp, _vp, C.c_int, _vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, C.c_int,
                                         _vp, C.c_int, _vp, _vp, _vp]),
    ("gat_b200_tfs_layer", C.c_int, [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                     _vp, _vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int, _vp]),
    ("gat_b200_tfs_online_counters", C.c_int, [_vp, C.c_int, _vp, _vp, C.c_int, _vp, _vp, _vp, _u64p, _vp]),
    ("gat_b200_check_device", C.c_int, []),
    ("gat_b200_device_alloc", C.c_int, [C.c_uint64, C.POINTER(_vp)]),
    ("gat_b200_device_free", C.c_int, [_vp]),
    ("gat_b200_copy_to_device", C.c_int, [_vp, _vp, C.c_uint64]),
    ("gat_b200_copy_to_host", C.c_int, [_vp, _vp, C.c_uint64]),
    ("gat_b200_model_create", C.c_int, [_vp, C.POINTER(_vp), C.c_int, C.POINTER(_vp)]),
    ("gat_b200_model_destroy", C.c_int, [_vp]),
    ("gat_b200_model_forward", C.c_int, [_vp, _vp, C.c_int, _vp, C.c_int, _vp]),
    ("gat_b200_model_enable_timing", C.c_int, [_vp, C.c_int]),
    ("gat_b200_model_stage_times", C.c_int, [_vp, _f32p]),
    ("gat_b200_model_launches", C.c_int, [_vp]),
    ("gat_b200_model_forward_async", C.c_int, [_vp, _vp, _vp, _vp]),
    ("gat_b200_model_join", C.c_int, [_vp, _vp]),
    ("gat_b200_peer_alloc", C.c_int, [C.c_uint64, C.POINTER(_vp), _vp]),
    ("gat_b200_peer_open", C.c_int, [_vp, C.POINTER(_vp)]),
    ("gat_b200_peer_close", C.c_int, [_vp]),
    ("gat_b200_peer_free", C.c_int, [_vp]),
    ("gat_b200_projection_scatter", C.c_int, [_vp, C.c_uint64, _vp, C.c_int, _vp, C.c_int, _vp, _vp, C.c_int,
                                              C.POINTER(_vp), C.POINTER(_vp), _vp]),
    ("gat_b200_peer_barrier", C.c_int, [C.POINTER(_vp), C.c_int, C.c_int, C.c_uint32, _vp]),
    ("gat_b200_copy_to_peers", C.c_int, [_vp, C.POINTER(_vp), C.c_int, C.c_uint64, C.POINTER(_vp)]),
    ("gat_b200_device_count", C.c_int, [C.POINTER(C.c_int)]),
    ("gat_b200_set_device", C.c_int, [C.c_int]),
    ("gat_b200_comm_id", C.c_int, [_vp]),
    ("gat_b200_comm_create", C.c_int, [_vp, C.c_int, C.c_int, C.POINTER(_vp)]),
    ("gat_b200_comm_create_file", C.c_int, [C.c_char_p, C.c_int, C.c_int, C.c_int, C.POINTER(_vp)]),
    ("gat_b200_comm_info", C.c_int, [_vp, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    ("gat_b200_comm_all_gather", C.c_int, [_vp, _vp, _vp, C.c_uint64]),
    ("gat_b200_comm_barrier", C.c_int, [_vp]),
    ("gat_b200_comm_destroy", C.c_int, [_vp]),
    ("gat_b200_partition", C.c_int, [C.c_uint64, _u64p, C.c_int, C.c_int, _u64p, _u64p, _u64p, _u64p]),
    ("gat_b200_partition_slots", C.c_int, [C.c_uint64, _u64p, C.c_int, C.c_int, C.c_uint64, _u32p, _u32p]),
    ("gat_b200_part_model_create", C.c_int, [_vp, C.c_uint64, _u64p, _u32p, C.POINTER(_vp), C.c_int, C.c_int, _vp,
                                             C.POINTER(_vp)]),
    ("gat_b200_part_model_rows", C.c_int, [_vp, _u64p, _u64p, _u64p]),
    ("gat_b200_part_model_forward", C.c_int, [_vp, _vp, C.c_int, _vp, C.c_int, _vp]),
    ("gat_b200_part_model_forward_async", C.c_int, [_vp, _vp, _vp, _vp]),
    ("gat_b200_part_model_join", C.c_int, [_vp, _vp]),
    ("gat_b200_part_model_enable_timing", C.c_int, [_vp, C.c_int]),
    ("gat_b200_part_model_stage_times", C.c_int, [_vp, _f32p]),
    ("gat_b200_part_model_launches", C.c_int, [_vp]),
    ("gat_b200_part_model_destroy", C.c_int, [_vp]),
    ("gat_b200_part_model_set_overlap", C.c_int, [_vp, C.c_int]),
    ("gat_b200_part_model_set_layer2_exchange", C.c_int, [_vp, C.c_int]),
]
for _name, _res, _args in SIGNATURES:
    _fn = getattr(_lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class GatError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def _check(rc: int):
    if rc != 0:
        raise GatError(rc, _lib.gat_b200_last_error().decode())


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def _ptr(t) -> Optional[int]:
    """Device pointer of a torch tensor (or int / None)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream(s) -> Optional[int]:
    if s is None:
        return None
    return s.cuda_stream if hasattr(s, "cuda_stream") else int(s)


def version() -> int:
    return _lib.gat_b200_version()


def padded_ld(width: int, dtype: int) -> int:
    return _lib.gat_b200_padded_ld(width, dtype)


# ---------------------------------------------------------------- host side
@dataclass
class Graph:
    """Destination-row CSR + FP32 features (baseline/include/gat.hpp:32-39)."""
    n: int
    e: int
    din: int
    classes: int
    row: np.ndarray  # u64 [n+1]
    col: np.ndarray  # u32 [e]
    x: np.ndarray    # f32 [n, din]

    def validate(self):
        _check(_lib.gat_b200_validate_csr(self.n, self.e, _p(self.row, _u64p), _p(self.col, _u32p)))
        if not np.isfinite(self.x).all():
            raise GatError(EINVAL, "nonfinite graph input")


@dataclass
class Param:
    """One layer (baseline/include/gat.hpp:42-47): W[in][heads*dim], aL, aR."""
    in_: int
    heads: int
    dim: int
    w: np.ndarray
    al: np.ndarray
    ar: np.ndarray

    @property
    def width(self) -> int:
        return self.heads * self.dim


def rne(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    _check(_lib.gat_b200_convert_host(_p(x, _f32p), _p(out, _u16p), x.size))
    return out


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def load_graph(path) -> Graph:
    n, e, d, c = C.c_uint64(), C.c_uint64(), C.c_uint32(), C.c_uint32()
    bpath = str(path).encode()
    _check(_lib.gat_b200_read_graph_header(bpath, C.byref(n), C.byref(e), C.byref(d), C.byref(c)))
    row = np.empty(n.value + 1, np.uint64)
    col = np.empty(max(e.value, 1), np.uint32)[: e.value]
    x = np.empty((n.value, d.value), np.float32)
    _check(_lib.gat_b200_read_graph(bpath, n.value, e.value, d.value, _p(row, _u64p), _p(col, _u32p), _p(x, _f32p)))
    return Graph(n.value, e.value, d.value, c.value, row, col, x)


def save_graph(g: Graph, path):
    _check(_lib.gat_b200_write_graph(str(path).encode(), g.n, g.e, g.din, g.classes,
                                     _p(np.ascontiguousarray(g.row, np.uint64), _u64p),
                                     _p(np.ascontiguousarray(g.col, np.uint32), _u32p),
                                     _p(np.ascontiguousarray(g.x, np.float32), _f32p)))


def model_shapes(din: int, classes: int):
    """Layer shapes of the reference model (baseline/src/common.cpp:53)."""
    return [(din, 8, 32), (256, 8, 32), (256, 1, classes)]


def _empty_model(din, classes) -> List[Param]:
    return [Param(i, h, d, np.empty((i, h * d), np.float32), np.empty(h * d, np.float32), np.empty(h * d, np.float32))
            for i, h, d in model_shapes(din, classes)]


def _arrays(model):
    arr = lambda xs: (_f32p * 3)(*[_p(x, _f32p) for x in xs])
    return arr([p.w for p in model]), arr([p.al for p in model]), arr([p.ar for p in model])


def random_model(din: int, classes: int, seed: int) -> List[Param]:
    """The reference's seeded untrained model (baseline/src/common.cpp:50-62)."""
    m = _empty_model(din, classes)
    _check(_lib.gat_b200_random_model(din, classes, seed, *_arrays(m)))
    return m


def glorot_model(din: int, classes: int, seed: int) -> List[Param]:
    """Glorot-uniform W (fan_in=in, fan_out=heads*dim) and a (fan = heads+dim)."""
    m = _empty_model(din, classes)
    for l, p in enumerate(m):
        lw = float(np.sqrt(6.0 / (p.in_ + p.width)))
        la = float(np.sqrt(6.0 / (p.heads + p.dim)))
        _check(_lib.gat_b200_synth_uniform(p.w.size, -lw, lw, seed, 100 + 3 * l, _p(p.w, _f32p)))
        _check(_lib.gat_b200_synth_uniform(p.width, -la, la, seed, 101 + 3 * l, _p(p.al, _f32p)))
        _check(_lib.gat_b200_synth_uniform(p.width, -la, la, seed, 102 + 3 * l, _p(p.ar, _f32p)))
    return m


def load_model(path, din: int, classes: int) -> List[Param]:
    m = _empty_model(din, classes)
    _check(_lib.gat_b200_read_weights(str(path).encode(), din, classes, *_arrays(m)))
    return m


def save_model(model: Sequence[Param], path):
    din, classes = model[0].in_, model[2].dim
    _check(_lib.gat_b200_write_weights(str(path).encode(), din, classes, *_arrays(model)))


def synth_uniform_graph(n: int, sources: int, seed: int):
    row = np.empty(n + 1, np.uint64)
    col = np.empty(n * (sources + 1), np.uint32)
    _check(_lib.gat_b200_synth_uniform_graph(n, sources, seed, _p(row, _u64p), _p(col, _u32p)))
    return row, col


def write_fixture(path, row, col, p: "Param", x, pw, den):
    """GATFIX1 fixed-p fixture (common.cpp:171-194): layer input x [n][in], p [e][heads], den [n][heads]."""
    row = np.ascontiguousarray(row, np.uint64)
    col = np.ascontiguousarray(col, np.uint32)
    n, e = len(row) - 1, len(col)
    f = lambda a: np.ascontiguousarray(a, np.float32)
    x, pw, den = f(x), f(pw), f(den)
    _check(_lib.gat_b200_write_fixture(str(path).encode(), n, e, p.in_, p.heads, p.dim, _p(row, _u64p),
                                       _p(col, _u32p), _p(f(p.w), _f32p), _p(f(p.al), _f32p), _p(f(p.ar), _f32p),
                                       _p(x, _f32p), _p(pw, _f32p), _p(den, _f32p)))


def read_fixture(path, row, col, p: "Param"):
    """Reads and validates a GATFIX1 fixture for this graph and layer: (x, p, den)."""
    row = np.ascontiguousarray(row, np.uint64)
    col = np.ascontiguousarray(col, np.uint32)
    n, e = len(row) - 1, len(col)
    x = np.empty((n, p.in_), np.float32)
    pw = np.empty((e, p.heads), np.float32)
    den = np.empty((n, p.heads), np.float32)
    f = lambda a: np.ascontiguousarray(a, np.float32)
    _check(_lib.gat_b200_read_fixture(str(path).encode(), n, e, p.in_, p.heads, p.dim, _p(row, _u64p),
                                      _p(col, _u32p), _p(f(p.w), _f32p), _p(f(p.al), _f32p), _p(f(p.ar), _f32p),
                                      _p(x, _f32p), _p(pw, _f32p), _p(den, _f32p)))
    return x, pw, den


def synth_powerlaw_graph(n: int, e: int, max_degree: int, gamma: float, seed: int):
    row = np.empty(n + 1, np.uint64)
    col = np.empty(e, np.uint32)
    _check(_lib.gat_b200_synth_powerlaw_graph(n, e, max_degree, gamma, seed, _p(row, _u64p), _p(col, _u32p)))
    return row, col


def synth_powerlaw_rowptr(n: int, e: int, max_degree: int, gamma: float, seed: int) -> np.ndarray:
    """The n+1 row pointers of synth_powerlaw_graph (no sources)."""
    row = np.empty(n + 1, np.uint64)
    _check(_lib.gat_b200_synth_powerlaw_rows(n, e, max_degree, gamma, seed, 0, 0, _p(row, _u64p), None))
    return row


def synth_powerlaw_cols(n: int, e: int, max_degree: int, gamma: float, seed: int, row: np.ndarray, r_lo: int,
                        r_hi: int) -> np.ndarray:
    """The sources of rows [r_lo, r_hi) of synth_powerlaw_graph."""
    row = np.ascontiguousarray(row, np.uint64).copy()
    col = np.empty(int(row[r_hi] - row[r_lo]), np.uint32)
    _check(_lib.gat_b200_synth_powerlaw_rows(n, e, max_degree, gamma, seed, r_lo, r_hi, _p(row, _u64p),
                                             _p(col, _u32p)))
    return col


def synth_rmat(log2_nodes: int, edges: int, a: float, b: float, c: float, seed: int, r_lo: int = 0,
               r_hi: Optional[int] = None, cols: bool = True):
    """RMAT graph generated on the current CUDA device: (row pointers of all
    rows, sources of rows [r_lo, r_hi) or None)."""
    n = 1 << log2_nodes
    r_hi = n if r_hi is None else r_hi
    row = np.empty(n + 1, np.uint64)
    e = C.c_uint64()
    _check(_lib.gat_b200_synth_rmat(log2_nodes, edges, a, b, c, seed, 0, 0, _p(row, _u64p), None, C.byref(e)))
    if not cols:
        return row, None
    col = np.empty(int(row[r_hi] - row[r_lo]), np.uint32)
    _check(_lib.gat_b200_synth_rmat(log2_nodes, edges, a, b, c, seed, r_lo, r_hi, _p(row, _u64p), _p(col, _u32p),
                                    C.byref(e)))
    return row, col


def synth_normal_range(offset: int, shape, seed: int, stream: int, scale: float = 1.0) -> np.ndarray:
    out = np.empty(shape, np.float32)
    _check(_lib.gat_b200_synth_normal_range(offset, out.size, scale, seed, stream, _p(out, _f32p)))
    return out


def synth_normal(shape, seed: int, stream: int, scale: float = 1.0) -> np.ndarray:
    out = np.empty(shape, np.float32)
    _check(_lib.gat_b200_synth_normal(out.size, scale, seed, stream, _p(out, _f32p)))
    return out


def synth_uniform(shape, lo: float, hi: float, seed: int, stream: int) -> np.ndarray:
    out = np.empty(shape, np.float32)
    _check(_lib.gat_b200_synth_uniform(out.size, lo, hi, seed, stream, _p(out, _f32p)))
    return out


# -------------------------------------------------------------- device side
class DeviceGraph:
    """CSR uploaded to the current CUDA device with its degree schedule."""

    def __init__(self, row: np.ndarray, col: np.ndarray, stream=None, n_src: Optional[int] = None):
        """n_src: number of source rows when the graph is a partition slice
        (gat_b200_graph_create_part); None for a square graph."""
        row = np.ascontiguousarray(row, np.uint64)
        col = np.ascontiguousarray(col, np.uint32)
        self.n = len(row) - 1
        self.e = len(col)
        h = _vp()
        if n_src is None:
            _check(_lib.gat_b200_graph_create(self.n, self.e, _p(row, _u64p), _p(col, _u32p), _stream(stream),
                                              C.byref(h)))
        else:
            _check(_lib.gat_b200_graph_create_part(self.n, n_src, self.e, _p(row, _u64p), _p(col, _u32p),
                                                   _stream(stream), C.byref(h)))
        self.handle = h

    def schedule(self):
        """(perm, neighbor_steps) as gat::degree_schedule (common.cpp:120-125)."""
        perm = np.empty(self.n, np.uint32)
        steps = C.c_uint64()
        _check(_lib.gat_b200_graph_schedule(self.handle, _p(perm, _u32p), C.byref(steps)))
        return perm, steps.value

    def info(self) -> dict:
        n, e = C.c_uint64(), C.c_uint64()
        md, nh, ns, se = C.c_uint32(), C.c_uint32(), C.c_uint32(), C.c_uint32()
        _check(_lib.gat_b200_graph_info(self.handle, C.byref(n), C.byref(e), C.byref(md), C.byref(nh),
                                        C.byref(ns), C.byref(se)))
        return dict(n=n.value, e=e.value, max_degree=md.value, n_hub=nh.value, n_seg=ns.value,
                    seg_edges=se.value)

    def close(self):
        if getattr(self, "handle", None):
            _lib.gat_b200_graph_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DeviceLayer:
    """Prepared layer parameters on the device (gat::prepare, common.cpp:97-119)."""

    def __init__(self, p: Param):
        self.param = p
        self.in_, self.heads, self.dim, self.width = p.in_, p.heads, p.dim, p.width
        h = _vp()
        w = np.ascontiguousarray(p.w, np.float32)
        al = np.ascontiguousarray(p.al, np.float32)
        ar = np.ascontiguousarray(p.ar, np.float32)
        _check(_lib.gat_b200_layer_create(p.in_, p.heads, p.dim, _p(w, _f32p), _p(al, _f32p), _p(ar, _f32p), C.byref(h)))
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            _lib.gat_b200_layer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def check_device():
    _check(_lib.gat_b200_check_device())


def convert(n, width, x, ld_in, out, ld_out, stream=None):
    _check(_lib.gat_b200_convert(n, width, _ptr(x), ld_in, _ptr(out), ld_out, _stream(stream)))


def projection(layer: DeviceLayer, n, x, ldx, precision, h=None, h_dtype=BF16, ldh=0, left=None, right=None,
               stream=None):
    _check(_lib.gat_b200_projection(layer.handle, n, _ptr(x), ldx, precision, _ptr(h), h_dtype, ldh, _ptr(left),
                                    _ptr(right), _stream(stream)))


PEER_HANDLE_BYTES = 64


def peer_alloc(nbytes: int):
    """(device pointer, IPC handle bytes) of a zero-filled allocation other
    processes of the node can map with peer_open."""
    ptr = C.c_void_p()
    h = C.create_string_buffer(PEER_HANDLE_BYTES)
    _check(_lib.gat_b200_peer_alloc(int(nbytes), C.byref(ptr), h))
    return int(ptr.value), bytes(h.raw)


def peer_open(handle: bytes) -> int:
    if len(handle) != PEER_HANDLE_BYTES:
        raise ValueError("peer handle must be 64 bytes")
    ptr = C.c_void_p()
    _check(_lib.gat_b200_peer_open(C.create_string_buffer(handle, PEER_HANDLE_BYTES), C.byref(ptr)))
    return int(ptr.value)


def peer_close(ptr: int):
    _check(_lib.gat_b200_peer_close(ptr))


def peer_free(ptr: int):
    _check(_lib.gat_b200_peer_free(ptr))


def projection_scatter(layer: DeviceLayer, n, x, ldx, h, ldh, left, right, h_peer, r_peer, stream=None):
    """BF16 projection of n rows storing H and R locally and into every peer
    table of h_peer / r_peer (device pointers, already offset to row 0)."""
    k = len(h_peer)
    if len(r_peer) != k:
        raise ValueError("h_peer and r_peer must have the same length")
    hp = (_vp * max(k, 1))(*[int(v) for v in h_peer])
    rp = (_vp * max(k, 1))(*[int(v) for v in r_peer])
    _check(_lib.gat_b200_projection_scatter(layer.handle, n, _ptr(x), ldx, _ptr(h), ldh, _ptr(left), _ptr(right),
                                            k, hp, rp, _stream(stream)))


def copy_to_peers(src: int, dsts, nbytes: int, streams):
    """dsts[j] <- src (nbytes) on streams[j] (copy engines)."""
    k = len(dsts)
    d = (_vp * max(k, 1))(*[int(v) for v in dsts])
    st = (_vp * max(k, 1))(*[_stream(v) for v in streams])
    _check(_lib.gat_b200_copy_to_peers(int(src), d, k, int(nbytes), st))


def peer_barrier(flags, rank: int, epoch: int, stream=None):
    """Cross-GPU barrier on `stream`; flags[j] = rank j's flag array."""
    arr = (_vp * len(flags))(*[int(v) for v in flags])
    _check(_lib.gat_b200_peer_barrier(arr, len(flags), rank, epoch & 0xFFFFFFFF, _stream(stream)))


def tfs_online_counters(g: DeviceGraph, heads, left, right, block, row_blocks=None, row_updates=None,
                        row_rescales=None, stream=None):
    """icpp_online's exact counters: totals (blocks, max_updates, rescales,
    rescale_events, neighbor_steps); per (row, head) arrays written to the
    given device uint64 buffers."""
    tot = np.zeros(5, np.uint64)
    _check(_lib.gat_b200_tfs_online_counters(g.handle, heads, _ptr(left), _ptr(right), block, _ptr(row_blocks),
                                             _ptr(row_updates), _ptr(row_rescales), _p(tot, _u64p),
                                             _stream(stream)))
    return tot


def max_prescan(g: DeviceGraph, heads, left, right, mx, stream=None):
    _check(_lib.gat_b200_max_prescan(g.handle, heads, _ptr(left), _ptr(right), _ptr(mx), _stream(stream)))


def edge_softmax(g: DeviceGraph, heads, left, right, p, den, score=None, mx=None, alpha=None, stream=None):
    """R0's edge softmax trace (ref_fp32.cpp:7-14): p [e][heads], den [n][heads],
    optionally score, the row maximum and alpha = p / den."""
    _check(_lib.gat_b200_edge_softmax(g.handle, heads, _ptr(left), _ptr(right), _ptr(score), _ptr(mx), _ptr(p),
                                      _ptr(den), _ptr(alpha), _stream(stream)))


def standard_aggregate(g: DeviceGraph, heads, dim, h, h_dtype, ldh, left, right, out, ldo, den, mx=None,
                       fixed_p=None, fixed_den=None, stream=None):
    _check(_lib.gat_b200_standard_aggregate(g.handle, heads, dim, _ptr(h), h_dtype, ldh, _ptr(left), _ptr(right),
                                            _ptr(fixed_p), _ptr(fixed_den), _ptr(out), ldo, _ptr(den), _ptr(mx),
                                            _stream(stream)))


def finish(n, heads, dim, den, hidden, out, ldo, stream=None):
    _check(_lib.gat_b200_finish(n, heads, dim, _ptr(den), int(hidden), _ptr(out), ldo, _stream(stream)))


def aggregate_fused(g: DeviceGraph, heads, dim, h, h_dtype, ldh, left, right, hidden, out, out_dtype, ldo,
                    stream=None):
    _check(_lib.gat_b200_aggregate_fused(g.handle, heads, dim, _ptr(h), h_dtype, ldh, _ptr(left), _ptr(right),
                                         int(hidden), _ptr(out), out_dtype, ldo, _stream(stream)))


def aggregate_fused_noalloc(n, e, row, col, heads, dim, h, h_dtype, ldh, left, right, hidden, out, out_dtype, ldo,
                            stream=None):
    """The fused aggregation without any device allocation (CSR given as device pointers)."""
    _check(_lib.gat_b200_aggregate_fused_noalloc(n, e, _ptr(row), _ptr(col), heads, dim, _ptr(h), h_dtype, ldh,
                                                 _ptr(left), _ptr(right), int(hidden), _ptr(out), out_dtype, ldo,
                                                 _stream(stream)))


def standard_layer(g: DeviceGraph, layer: DeviceLayer, x, ldx, path, hidden, h, left, right, out, out_dtype, ldo,
                   stream=None):
    _check(_lib.gat_b200_standard_layer(g.handle, layer.handle, _ptr(x), ldx, path, int(hidden), _ptr(h), _ptr(left),
                                        _ptr(right), _ptr(out), out_dtype, ldo, _stream(stream)))


def lr_reordered(layer: DeviceLayer, n, x, x_dtype, ldx, policy, left, right, x_bf16=None, ld_bf16=0, stream=None):
    """[L|R] = X . (W a) (baseline_standard.cpp:29-43), optionally writing the BF16 copy of X."""
    _check(_lib.gat_b200_lr_reordered(layer.handle, n, _ptr(x), x_dtype, ldx, policy, _ptr(x_bf16), ld_bf16,
                                      _ptr(left), _ptr(right), _stream(stream)))


def tfs_aggregate(g: DeviceGraph, layer: DeviceLayer, x, ldx, left, right, out, ldo, den, mx=None, rounding=TFS_EDGE,
                  block=0, threshold=1, fixed_p=None, fixed_den=None, max_out=None, stream=None):
    """TFS aggregation (baseline_tfs.cpp:16-110 and the icpp_* variants): unnormalized V, den (, max)."""
    _check(_lib.gat_b200_tfs_aggregate(g.handle, layer.handle, _ptr(x), ldx, _ptr(left), _ptr(right), _ptr(mx),
                                       _ptr(fixed_p), _ptr(fixed_den), rounding, block, threshold, _ptr(out), ldo,
                                       _ptr(den), _ptr(max_out), _stream(stream)))


def tfs_layer(g: DeviceGraph, layer: DeviceLayer, x, x_dtype, ldx, hidden, x_bf16, left, right, mx, den, out,
              out_dtype, ldo, policy=LR_BF16, rounding=TFS_EDGE, block=0, threshold=1, stream=None):
    """One TFS layer (baseline_tfs.cpp:111-117 / icpp_*::layer)."""
    _check(_lib.gat_b200_tfs_layer(g.handle, layer.handle, _ptr(x), x_dtype, ldx, int(hidden), policy, rounding, block,
                                   threshold, _ptr(x_bf16), _ptr(left), _ptr(right), _ptr(mx), _ptr(den), _ptr(out),
                                   out_dtype, ldo, _stream(stream)))


class DeviceModel:
    """The three-layer forward (bench/main.cpp:171-172) with all buffers preallocated."""

    def __init__(self, g: DeviceGraph, layers: Sequence[DeviceLayer], path: int = PATH_STANDARD_BF16):
        self.g = g
        self.layers = list(layers)
        arr = (_vp * 3)(*[l.handle for l in self.layers])
        h = _vp()
        _check(_lib.gat_b200_model_create(g.handle, arr, path, C.byref(h)))
        self.handle = h
        self.classes = self.layers[2].width
        self.din = self.layers[0].in_

    def forward(self, x, logits, x_on_host: bool, logits_on_host: bool, stream=None):
        """x, logits: torch tensors (pinned host or device) or raw pointers."""
        _check(_lib.gat_b200_model_forward(self.handle, _ptr(x), int(x_on_host), _ptr(logits), int(logits_on_host),
                                           _stream(stream)))

    def forward_async(self, x_host, logits_host, stream=None):
        """Pipelined host-to-host forward (see gat_b200_model_forward_async); pinned host tensors."""
        _check(_lib.gat_b200_model_forward_async(self.handle, _ptr(x_host), _ptr(logits_host), _stream(stream)))

    def join(self, stream=None):
        """Make `stream` wait for every submitted forward_async (no host block)."""
        _check(_lib.gat_b200_model_join(self.handle, _stream(stream)))

    STAGES = ("h2d", "convert", "projection_l1", "aggregate_l1", "projection_l2", "aggregate_l2",
              "projection_l3", "aggregate_l3", "d2h")

    def enable_timing(self, steps: int):
        _check(_lib.gat_b200_model_enable_timing(self.handle, steps))
        self._timing_steps = steps

    def stage_times(self) -> np.ndarray:
        """[sets, 9] milliseconds per stage (see STAGES)."""
        buf = np.zeros((max(1, self._timing_steps), len(self.STAGES)), np.float32)
        k = _lib.gat_b200_model_stage_times(self.handle, _p(buf, _f32p))
        if k < 0:
            _check(k)
        return buf[:k]

    def launches(self) -> int:
        return _lib.gat_b200_model_launches(self.handle)

    def close(self):
        if getattr(self, "handle", None):
            _lib.gat_b200_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------- multi-GPU
COMM_ID_BYTES = 128
EXCHANGE_P2P, EXCHANGE_NCCL = 0, 1
PART_STAGES = ("h2d", "input_exchange", "barrier_l1", "projection_l1", "aggregate_l1", "projection_l2",
               "barrier_l2", "aggregate_l2", "projection_l3", "barrier_l3", "aggregate_l3", "d2h")


def comm_id() -> bytes:
    """A fresh NCCL unique id (rank 0 makes it, every rank passes it to Comm)."""
    b = C.create_string_buffer(COMM_ID_BYTES)
    _check(_lib.gat_b200_comm_id(b))
    return b.raw


def partition(row: np.ndarray, world: int, chunks: int = 1):
    """(cuts[world+1], chunk_cuts[world, chunks+1], block_rows, table_rows) of the partitioned forward."""
    row = np.ascontiguousarray(row, np.uint64)
    n = len(row) - 1
    cuts = np.zeros(world + 1, np.uint64)
    cc = np.zeros(world * (chunks + 1), np.uint64)
    br, tr = C.c_uint64(), C.c_uint64()
    _check(_lib.gat_b200_partition(n, _p(row, _u64p), world, chunks, _p(cuts, _u64p), _p(cc, _u64p), C.byref(br),
                                   C.byref(tr)))
    return cuts.astype(np.int64), cc.reshape(world, chunks + 1).astype(np.int64), int(br.value), int(tr.value)


def partition_slots(row: np.ndarray, world: int, chunks: int, src: np.ndarray) -> np.ndarray:
    """Table rows of global source ids under partition(row, world, chunks)."""
    row = np.ascontiguousarray(row, np.uint64)
    src = np.ascontiguousarray(src, np.uint32)
    out = np.empty(len(src), np.uint32)
    _check(_lib.gat_b200_partition_slots(len(row) - 1, _p(row, _u64p), world, chunks, len(src), _p(src, _u32p),
                                         _p(out, _u32p)))
    return out


class Comm:
    """The node's communicator (gat_b200_comm_create): rank `rank` of `world`
    on the current device, joined with rank 0's unique id (or through `path`)."""

    def __init__(self, world: int, rank: int, uid: Optional[bytes] = None, path: Optional[str] = None,
                 timeout_ms: int = 60000):
        h = _vp()
        if path is not None:
            _check(_lib.gat_b200_comm_create_file(str(path).encode(), world, rank, timeout_ms, C.byref(h)))
        else:
            buf = C.create_string_buffer(uid, COMM_ID_BYTES) if uid is not None else None
            _check(_lib.gat_b200_comm_create(buf, world, rank, C.byref(h)))
        self.handle = h
        self.world, self.rank = world, rank

    def all_gather(self, blob: bytes) -> List[bytes]:
        out = C.create_string_buffer(len(blob) * self.world)
        _check(_lib.gat_b200_comm_all_gather(self.handle, C.create_string_buffer(blob, len(blob)), out, len(blob)))
        return [out.raw[j * len(blob):(j + 1) * len(blob)] for j in range(self.world)]

    def barrier(self):
        _check(_lib.gat_b200_comm_barrier(self.handle))

    def close(self):
        if getattr(self, "handle", None):
            _lib.gat_b200_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PartModel:
    """The row-partitioned three-layer forward of this rank
    (gat_b200_part_model_*): row = all n+1 row pointers, col_rows = the
    sources of this rank's rows (see rows())."""

    def __init__(self, comm: Comm, row: np.ndarray, col_rows: np.ndarray, layers: Sequence[DeviceLayer],
                 exchange: int = EXCHANGE_P2P, chunks: int = 1, stream=None):
        row = np.ascontiguousarray(row, np.uint64)
        col_rows = np.ascontiguousarray(col_rows, np.uint32)
        self.layers = list(layers)
        arr = (_vp * 3)(*[l.handle for l in self.layers])
        h = _vp()
        _check(_lib.gat_b200_part_model_create(comm.handle, len(row) - 1, _p(row, _u64p), _p(col_rows, _u32p), arr,
                                               exchange, chunks, _stream(stream), C.byref(h)))
        self.handle = h
        self.comm = comm
        self.classes = self.layers[2].width
        self.din = self.layers[0].in_
        self.lo, self.hi, self.e_loc = self.rows()
        self.n_loc = self.hi - self.lo

    def rows(self):
        lo, hi, e = C.c_uint64(), C.c_uint64(), C.c_uint64()
        _check(_lib.gat_b200_part_model_rows(self.handle, C.byref(lo), C.byref(hi), C.byref(e)))
        return int(lo.value), int(hi.value), int(e.value)

    def forward(self, x, logits, x_on_host: bool, logits_on_host: bool, stream=None):
        _check(_lib.gat_b200_part_model_forward(self.handle, _ptr(x), int(x_on_host), _ptr(logits),
                                                int(logits_on_host), _stream(stream)))

    def forward_async(self, x_host, logits_host, stream=None):
        _check(_lib.gat_b200_part_model_forward_async(self.handle, _ptr(x_host), _ptr(logits_host), _stream(stream)))

    def join(self, stream=None):
        _check(_lib.gat_b200_part_model_join(self.handle, _stream(stream)))

    def enable_timing(self, on: bool):
        _check(_lib.gat_b200_part_model_enable_timing(self.handle, int(on)))

    def stage_times(self) -> dict:
        buf = np.zeros(len(PART_STAGES), np.float32)
        _check(_lib.gat_b200_part_model_stage_times(self.handle, _p(buf, _f32p)))
        return {k: float(v) for k, v in zip(PART_STAGES, buf)}

    def launches(self) -> int:
        return _lib.gat_b200_part_model_launches(self.handle)

    def set_overlap(self, reserved_sms: int):
        """SMs left to the exchange while a chunk aggregates (0: no overlap)."""
        _check(_lib.gat_b200_part_model_set_overlap(self.handle, reserved_sms))

    def set_layer2_exchange(self, inputs: bool):
        """True: layer 2's input rows travel in the layer-1 aggregation's epilogue
        and every rank projects the whole table; False: the layer-2 projection
        stores H and R into every rank's table."""
        _check(_lib.gat_b200_part_model_set_layer2_exchange(self.handle, int(inputs)))

    def close(self):
        """Collective: every rank calls it."""
        if getattr(self, "handle", None):
            h, self.handle = self.handle, None
            _check(_lib.gat_b200_part_model_destroy(h))
