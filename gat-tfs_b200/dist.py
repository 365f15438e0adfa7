"""Row-partitioned multi-GPU forward: one process per GPU, NCCL over NVLink.

Destination rows are cut into contiguous ranges balanced by edge count: rank k
owns rows [cuts[k], cuts[k+1]) with cuts[k] the first row whose CSR offset
reaches k*E/G. Destination rows are independent given the projected features
of all their sources, so each layer is

  1. projection of the rank's own rows (tcgen05 kernel): H_k, L_k, R_k;
  2. one all-gather of H (and of R) into every rank's feature table;
  3. edge-softmax aggregation of the rank's own rows from that table.

The all-gather is the only exchange. Ranks own different row counts while
ncclAllGather moves equal blocks, so every rank's block is padded to the
largest row count n_max, and the column ids of the rank's CSR slice are
remapped once into that padded table: source s of rank r's range becomes
r*n_max + (s - cuts[r]).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import numpy as np

import gatb200 as G


def partition(row: np.ndarray, world: int) -> np.ndarray:
    """Row cut points (length world+1) balancing the edge count per rank."""
    row = np.asarray(row, np.uint64)
    n = len(row) - 1
    e = int(row[-1])
    targets = [(k * e) // world for k in range(1, world)]
    inner = np.searchsorted(row, np.asarray(targets, np.uint64), side="left").astype(np.int64)
    cuts = np.concatenate([[0], np.clip(inner, 0, n), [n]]).astype(np.int64)
    return np.maximum.accumulate(cuts)


def slice_local(row: np.ndarray, col_rows: np.ndarray, cuts: np.ndarray, rank: int):
    """CSR slice of `rank` from the global row pointers and the sources of the
    rank's own rows (col[row[lo]:row[hi]]), with the source ids remapped into
    the padded feature table. Returns (row_loc u64[n_loc+1], col_loc u32, n_max)."""
    row = np.asarray(row, np.uint64)
    n_max = int(np.diff(cuts).max())
    lo, hi = int(cuts[rank]), int(cuts[rank + 1])
    b = int(row[lo])
    if len(col_rows) != int(row[hi]) - b:
        raise ValueError("col_rows must hold the sources of the rank's rows")
    row_loc = (row[lo:hi + 1] - np.uint64(b)).astype(np.uint64)
    src = np.asarray(col_rows).astype(np.int64)
    owner = np.searchsorted(cuts, src, side="right") - 1
    col_loc = (owner * n_max + (src - cuts[owner])).astype(np.uint32)
    return row_loc, col_loc, n_max


def slice_graph(row: np.ndarray, col: np.ndarray, cuts: np.ndarray, rank: int):
    """slice_local from the whole column array."""
    lo, hi = int(cuts[rank]), int(cuts[rank + 1])
    return slice_local(row, np.asarray(col)[int(row[lo]):int(row[hi])], cuts, rank)


class PartitionedModel:
    """Three-layer BF16 forward of this rank's rows (bench/main.cpp:171-172 per rank)."""

    def __init__(self, row: np.ndarray, col_rows: np.ndarray, params: Sequence[G.Param], rank: int, world: int,
                 stream=None, dist_module=None, cuts: Optional[np.ndarray] = None):
        """row: all n+1 row pointers; col_rows: the sources of this rank's rows
        (col[row[cuts[rank]]:row[cuts[rank+1]]]); cuts: partition(row, world)."""
        import torch
        self.torch = torch
        self.dist = dist_module
        self.rank, self.world = rank, world
        self.cuts = partition(row, world) if cuts is None else cuts
        row_loc, col_loc, n_max = slice_local(row, col_rows, self.cuts, rank)
        self.n_loc = len(row_loc) - 1
        self.e_loc = len(col_loc)
        self.n_max = n_max
        self.stream = stream
        self.g = G.DeviceGraph(row_loc, col_loc, stream, n_src=world * n_max)
        self.layers = [G.DeviceLayer(p) for p in params]
        self.din = params[0].in_
        self.classes = params[2].width
        dev = torch.device("cuda", torch.cuda.current_device())
        wmax = max(p.width for p in params)
        ldh_max = G.padded_ld(wmax, G.BF16)
        self.ld0 = G.padded_ld(self.din, G.BF16)
        self.ld_hidden = G.padded_ld(max(params[0].width, params[1].width), G.BF16)
        n = self.n_loc
        i16 = torch.int16
        self.x_f32 = torch.empty((n, self.din), dtype=torch.float32, device=dev)
        self.x0 = torch.zeros((n, self.ld0), dtype=i16, device=dev)
        self.h_send = torch.zeros((n_max * ldh_max,), dtype=i16, device=dev)
        self.h_full = torch.zeros((world * n_max * ldh_max,), dtype=i16, device=dev)
        self.r_send = torch.zeros((n_max * 8,), dtype=torch.float32, device=dev)
        self.r_full = torch.zeros((world * n_max * 8,), dtype=torch.float32, device=dev)
        self.left = torch.zeros((n * 8,), dtype=torch.float32, device=dev)
        self.xs = [torch.zeros((n, self.ld_hidden), dtype=i16, device=dev) for _ in range(2)]
        self.logits = torch.empty((n, self.classes), dtype=torch.float32, device=dev)
        self.events = None

    def enable_timing(self, on: bool):
        torch = self.torch
        self.events = [torch.cuda.Event(enable_timing=True) for _ in range(12)] if on else None
        self.stage_ms: List[np.ndarray] = []

    def _mark(self, i):
        # events 0 start, 1 after the input copy, 2+3l / 3+3l / 4+3l before the
        # projection / all-gather / aggregation of layer l, 11 end
        if self.events is not None:
            self.events[i].record(self.torch.cuda.current_stream())

    def forward(self, x, logits, x_on_host: bool, logits_on_host: bool):
        """x: this rank's FP32 input rows [n_loc, din]; logits: [n_loc, classes]."""
        torch = self.torch
        n = self.n_loc
        self._mark(0)
        xin = x
        if x_on_host:
            self.x_f32.copy_(x, non_blocking=True)
            xin = self.x_f32
        self._mark(1)
        G.convert(n, self.din, xin, self.din, self.x0, self.ld0, self.stream)
        lin, ldin = self.x0, self.ld0
        for l, p in enumerate(self.layers):
            ldh = G.padded_ld(p.width, G.BF16)
            K = p.heads
            hs = self.h_send[: self.n_max * ldh]
            hf = self.h_full[: self.world * self.n_max * ldh]
            rs = self.r_send[: self.n_max * K]
            rf = self.r_full[: self.world * self.n_max * K]
            self._mark(2 + 3 * l)
            G.projection(p, n, lin, ldin, G.BF16, hs, G.BF16, ldh, self.left, rs, self.stream)
            self._mark(3 + 3 * l)
            if self.world > 1:
                # the feature tables hold BF16 bit patterns in int16 storage; NCCL
                # has no 16-bit integer type, so the exchange goes through a
                # bfloat16 view of the same bytes
                self.dist.all_gather_into_tensor(hf.view(torch.bfloat16), hs.view(torch.bfloat16))
                self.dist.all_gather_into_tensor(rf, rs)
            else:
                hf, rf = hs, rs
            self._mark(4 + 3 * l)
            last = l == 2
            if last:
                dst = logits if not logits_on_host else self.logits
                G.aggregate_fused(self.g, K, p.dim, hf, G.BF16, ldh, self.left, rf, False, dst, G.F32, p.width,
                                  self.stream)
            else:
                dst = self.xs[l]
                G.aggregate_fused(self.g, K, p.dim, hf, G.BF16, ldh, self.left, rf, True, dst, G.BF16,
                                  self.ld_hidden, self.stream)
                lin, ldin = dst, self.ld_hidden
        self._mark(11)
        if logits_on_host:
            logits.copy_(self.logits, non_blocking=True)

    def stage_times(self) -> dict:
        """ms of the last forward: projection, all-gather and aggregation per layer."""
        torch = self.torch
        torch.cuda.synchronize()
        ev = self.events
        out = {}
        for l in range(3):
            out[f"projection_l{l + 1}"] = ev[2 + 3 * l].elapsed_time(ev[3 + 3 * l])
            out[f"allgather_l{l + 1}"] = ev[3 + 3 * l].elapsed_time(ev[4 + 3 * l])
            nxt = ev[5 + 3 * l] if l < 2 else ev[11]
            out[f"aggregate_l{l + 1}"] = ev[4 + 3 * l].elapsed_time(nxt)
        return out

    def close(self):
        for l in self.layers:
            l.close()
        self.g.close()
