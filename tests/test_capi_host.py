"""C-ABI boundary and host logic of libgat_b200.so (no GPU needed)."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

import gatb200 as G
import oracle as O
from conftest import cuda_available

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "gat_b200.h").read_text()
    return sorted(set(re.findall(r"\b(gat_b200_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(str(G.LIB_PATH))
    names = declared_symbols()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding declares a signature for each of them
    bound = {s[0] for s in G.SIGNATURES}
    assert set(names) <= bound, set(names) - bound


def test_version_and_padded_ld():
    assert G.version() >= 100
    assert G.padded_ld(256, G.BF16) == 256
    assert G.padded_ld(47, G.BF16) == 48
    assert G.padded_ld(47, G.F32) == 48
    assert G.padded_ld(100, G.BF16) == 104
    assert G.padded_ld(7, G.F32) == 8


def test_host_rne_matches_oracle():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.normal(0, 3, 100000).astype(np.float32),
                        np.array([0.0, -0.0, np.inf, -np.inf, 3.4e38, -3.4e38, 1e-40, np.nan], np.float32),
                        (np.arange(4096, dtype=np.uint32) * 0x10001 + 0x3F808000).view(np.float32)])
    got = G.rne(x)
    want = np.array([O.rne(float(v)) for v in x], np.uint16)
    finite = np.isfinite(x)
    assert np.array_equal(got[finite], want[finite])
    assert np.array_equal(got[~finite & ~np.isnan(x)], want[~finite & ~np.isnan(x)])
    # NaN stays a quiet NaN
    assert (got[np.isnan(x)] & 0x7FC0 == 0x7FC0).all()


def _good_graph():
    row = np.array([0, 2, 3, 3, 6], np.uint64)
    col = np.array([1, 2, 0, 0, 1, 3], np.uint32)
    return row, col


def test_validate_csr_accepts_and_rejects():
    # The reference's negative tests (baseline/tests/boundaries.cpp:54-59).
    row, col = _good_graph()
    G.Graph(4, 6, 1, 1, row, col, np.zeros((4, 1), np.float32)).validate()
    bad = row.copy()
    bad[2] = 7
    with pytest.raises(G.GatError, match="nonmonotone CSR"):
        G.Graph(4, 6, 1, 1, bad, col, np.zeros((4, 1), np.float32)).validate()
    badc = col.copy()
    badc[0] = 4
    with pytest.raises(G.GatError, match="source index out of bounds"):
        G.Graph(4, 6, 1, 1, row, badc, np.zeros((4, 1), np.float32)).validate()
    badb = row.copy()
    badb[-1] = 5
    with pytest.raises(G.GatError, match="bad CSR bounds"):
        G.Graph(4, 6, 1, 1, badb, col, np.zeros((4, 1), np.float32)).validate()
    x = np.zeros((4, 1), np.float32)
    x[0, 0] = np.nan
    with pytest.raises(G.GatError, match="nonfinite"):
        G.Graph(4, 6, 1, 1, row, col, x).validate()


def test_gatbin_and_gatwgt_round_trip(tmp_path):
    row, col = _good_graph()
    x = np.arange(12, dtype=np.float32).reshape(4, 3)
    g = G.Graph(4, 6, 3, 2, row, col, x)
    G.save_graph(g, tmp_path / "g.gatbin")
    h = G.load_graph(tmp_path / "g.gatbin")
    assert (h.n, h.e, h.din, h.classes) == (4, 6, 3, 2)
    assert np.array_equal(h.row, row) and np.array_equal(h.col, col) and np.array_equal(h.x, x)
    m = G.random_model(3, 2, 5)
    G.save_model(m, tmp_path / "w.gatwgt")
    m2 = G.load_model(tmp_path / "w.gatwgt", 3, 2)
    for a, b in zip(m, m2):
        assert np.array_equal(a.w, b.w) and np.array_equal(a.al, b.al) and np.array_equal(a.ar, b.ar)
    with pytest.raises(G.GatError, match="checkpoint model shape mismatch"):
        G.load_model(tmp_path / "w.gatwgt", 4, 2)
    (tmp_path / "bad.gatbin").write_bytes(b"GATBIN2\0" + b"\0" * 24)
    with pytest.raises(G.GatError, match="bad graph magic"):
        G.load_graph(tmp_path / "bad.gatbin")
    data = (tmp_path / "g.gatbin").read_bytes()
    (tmp_path / "trunc.gatbin").write_bytes(data[:-8])
    with pytest.raises(G.GatError, match="truncated"):
        G.load_graph(tmp_path / "trunc.gatbin")


def test_layer_create_validates_shapes():
    # Param::validate (baseline/src/common.cpp:45-49) before any device work.
    p = G.Param(4, 9, 2, np.zeros((4, 18), np.float32), np.zeros(18, np.float32), np.zeros(18, np.float32))
    with pytest.raises(G.GatError, match="heads <=8"):
        G.DeviceLayer(p)
    p = G.Param(4, 1, 65, np.zeros((4, 65), np.float32), np.zeros(65, np.float32), np.zeros(65, np.float32))
    with pytest.raises(G.GatError, match="head_dim <=64"):
        G.DeviceLayer(p)
    w = np.zeros((4, 8), np.float32)
    w[1, 1] = np.inf
    p = G.Param(4, 1, 8, w, np.zeros(8, np.float32), np.zeros(8, np.float32))
    with pytest.raises(G.GatError, match="nonfinite W"):
        G.DeviceLayer(p)


def test_synthetic_generators():
    row, col = G.synth_uniform_graph(64, 7, 3)
    deg = np.diff(row.astype(np.int64))
    assert np.all(deg == 8)
    for i in range(64):
        r = col[row[i]:row[i + 1]]
        assert i in r and len(np.unique(r)) == 8 and np.all(np.diff(r.astype(np.int64)) > 0)
    row, col = G.synth_powerlaw_graph(5000, 60000, 1500, 2.1, 9)
    deg = np.diff(row.astype(np.int64))
    assert row[-1] == 60000 and deg.max() == 1500 and deg.min() >= 2
    r2, c2 = G.synth_powerlaw_graph(5000, 60000, 1500, 2.1, 9)
    assert np.array_equal(row, r2) and np.array_equal(col, c2)
    x = G.synth_normal((1000, 10), 1, 1)
    assert abs(float(x.mean())) < 0.05 and abs(float(x.std()) - 1) < 0.05


@pytest.mark.skipif(cuda_available(), reason="checks the no-GPU error path")
def test_device_calls_fail_cleanly_without_gpu():
    row, col = _good_graph()
    with pytest.raises(G.GatError) as e:
        G.DeviceGraph(row, col)
    assert e.value.code == G.ECUDA


def test_multi_gpu_and_rmat_entry_points_validate_arguments():
    """Argument checks of the peer-memory, scatter and RMAT entry points happen
    before any CUDA call (status GAT_B200_EINVAL = 1 and the message)."""
    lib = G._lib
    vp = C.c_void_p
    flags = (vp * 9)(*([1] * 9))
    assert lib.gat_b200_peer_barrier(flags, 9, 0, 1, None) == 1
    assert "world size must be 1..8" in lib.gat_b200_last_error().decode()
    assert lib.gat_b200_peer_barrier(flags, 2, 2, 1, None) == 1
    assert "rank outside the world" in lib.gat_b200_last_error().decode()
    assert lib.gat_b200_peer_barrier(None, 2, 0, 1, None) == 1
    assert lib.gat_b200_peer_barrier(flags, 1, 0, 1, None) == 0  # one rank: nothing to wait for
    assert lib.gat_b200_copy_to_peers(vp(1), flags, 8, 16, flags) == 1
    assert "ndst must be 0..7" in lib.gat_b200_last_error().decode()
    assert lib.gat_b200_copy_to_peers(None, flags, 0, 16, flags) == 0  # no destinations
    assert lib.gat_b200_projection_scatter(None, 10, vp(1), 16, vp(1), 16, None, vp(1), 0, None, None, None) == 1
    assert "null argument" in lib.gat_b200_last_error().decode()
    assert lib.gat_b200_peer_alloc(16, None, None) == 1
    assert lib.gat_b200_peer_open(None, None) == 1
    assert lib.gat_b200_peer_close(None) == 0 and lib.gat_b200_peer_free(None) == 0
    row = np.zeros(5, np.uint64)
    rp = row.ctypes.data_as(C.POINTER(C.c_uint64))
    assert lib.gat_b200_synth_rmat(2, 10, 0.5, 0.3, 0.3, 1, 0, 0, rp, None, None) == 1
    assert "a+b+c < 1" in lib.gat_b200_last_error().decode()
    assert lib.gat_b200_synth_rmat(0, 10, 0.57, 0.19, 0.19, 1, 0, 0, rp, None, None) == 1
    assert lib.gat_b200_synth_rmat(2, 10, 0.57, 0.19, 0.19, 1, 3, 2, rp, None, None) == 1
    assert "bad row range" in lib.gat_b200_last_error().decode()
    assert lib.gat_b200_synth_rmat(30, 1 << 31, 0.57, 0.19, 0.19, 1, 0, 0, rp, None, None) == 1


def test_edge_softmax_validates_arguments():
    """gat_b200_edge_softmax's checks come before any CUDA call."""
    lib = G._lib
    vp = C.c_void_p
    assert lib.gat_b200_edge_softmax(None, 8, vp(1), vp(1), None, None, vp(1), vp(1), None, None) == 1
    assert "edge_softmax: null buffer" in lib.gat_b200_last_error().decode()
    assert lib.gat_b200_edge_softmax(vp(1), 8, vp(1), vp(1), None, None, None, vp(1), None, None) == 1
    assert "edge_softmax: null buffer" in lib.gat_b200_last_error().decode()
    assert lib.gat_b200_edge_softmax(vp(1), 9, vp(1), vp(1), None, None, vp(1), vp(1), None, None) == 1
    assert "invalid parameter shape" in lib.gat_b200_last_error().decode()


def test_bindings_match_header_arity():
    """Every ctypes binding in gatb200.py takes as many arguments as the C
    declaration in include/gat_b200.h, and every declared function is bound."""
    import re
    hdr = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "gat_b200.h").read_text(), flags=re.S)
    decls = {}
    for m in re.finditer(r"\b(gat_b200_\w+)\s*\(([^;{]*?)\)\s*;", hdr):
        args = m.group(2).strip()
        decls[m.group(1)] = 0 if args in ("", "void") else len(args.split(","))
    src = (ROOT / "gat-tfs_b200" / "gatb200.py").read_text()
    bound = {}
    for m in re.finditer(r'\("(gat_b200_\w+)",\s*[^\[]+?,\s*\[([^\]]*)\]\)', src, flags=re.S):
        bound[m.group(1)] = len([a for a in m.group(2).split(",") if a.strip()])
    assert decls and set(decls) == set(bound), sorted(set(decls) ^ set(bound))
    assert {k: v for k, v in bound.items() if decls[k] != v} == {}
