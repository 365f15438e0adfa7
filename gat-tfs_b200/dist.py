"""Python statement of the row partition of the multi-GPU forward.

The partitioned forward itself is native: gat_b200_part_model_* in the
library (gat-tfs_b200/csrc/part.cu), with its layout computed by
gat_b200_partition. This module states the same layout in numpy for the CPU
multi-process runs (gloo ranks running the oracle through the identical
chunk-major table, tests/test_dist_cpu.py), and tests/test_partition.py
checks that both give the same cuts, blocks and table rows bit for bit.

Destination rows are cut into contiguous ranges balanced by edge count: rank
k owns rows [cuts[k], cuts[k+1]) with cuts[k] the first row whose CSR offset
reaches k*E/G. Rows of a rank may be cut into `chunks` row chunks (balanced by
edges). The feature table is chunk-major with equal blocks: chunk c of every
rank is padded to the largest chunk (chunk_max rows, a multiple of 4) and the
table holds, for c = 0..chunks-1, the chunk-c blocks of ranks 0..G-1 one
after the other. Source s, owned by rank r at local chunk c and offset i, sits
at table row (c*G + r)*chunk_max + i.
"""
from __future__ import annotations

from typing import Optional

import numpy as np


def partition(row: np.ndarray, world: int) -> np.ndarray:
    """Row cut points (length world+1) balancing the edge count per rank."""
    row = np.asarray(row, np.uint64)
    n = len(row) - 1
    e = int(row[-1])
    targets = [(k * e) // world for k in range(1, world)]
    inner = np.searchsorted(row, np.asarray(targets, np.uint64), side="left").astype(np.int64)
    cuts = np.concatenate([[0], np.clip(inner, 0, n), [n]]).astype(np.int64)
    return np.maximum.accumulate(cuts)


class Layout:
    """Rank cuts, per-rank chunk cuts and the chunk-major feature table."""

    def __init__(self, row: np.ndarray, world: int, chunks: int, cuts: Optional[np.ndarray] = None):
        row = np.asarray(row, np.uint64)
        self.world, self.chunks = world, chunks
        self.cuts = partition(row, world) if cuts is None else np.asarray(cuts, np.int64)
        cc = np.empty((world, chunks + 1), np.int64)
        for r in range(world):
            lo, hi = int(self.cuts[r]), int(self.cuts[r + 1])
            sub = row[lo:hi + 1]
            e0, e1 = int(sub[0]), int(sub[-1])
            targets = np.asarray([e0 + (k * (e1 - e0)) // chunks for k in range(1, chunks)], np.uint64)
            inner = lo + np.searchsorted(sub, targets, side="left").astype(np.int64)
            cc[r] = np.maximum.accumulate(np.concatenate([[lo], np.clip(inner, lo, hi), [hi]]))
        self.ccuts = cc  # global row boundaries [world, chunks+1]
        # padded to 4 rows so every block of an FP32 table starts 16-byte aligned
        self.chunk_max = (max(1, int(np.diff(cc, axis=1).max())) + 3) // 4 * 4
        self.n_table = chunks * world * self.chunk_max
        self._starts = cc[:, :-1].reshape(-1)  # ascending: ranks' ranges are contiguous

    def slots(self, src: np.ndarray) -> np.ndarray:
        """Table rows of global source ids."""
        src = np.asarray(src).astype(np.int64)
        k = np.searchsorted(self._starts, src, side="right") - 1  # rank*chunks + chunk (empty chunks skipped)
        r, c = k // self.chunks, k % self.chunks
        return ((c * self.world + r) * self.chunk_max + (src - self._starts[k])).astype(np.uint32)

    def chunk_rows(self, rank: int, c: int):
        """(first, end) local row of chunk c of `rank`."""
        lo = int(self.cuts[rank])
        return int(self.ccuts[rank, c]) - lo, int(self.ccuts[rank, c + 1]) - lo

    def slice_chunk(self, row: np.ndarray, col_rows: np.ndarray, rank: int, c: int):
        """CSR slice of chunk c of `rank` with sources remapped to table rows.
        col_rows: the sources of all of the rank's rows (col[row[lo]:row[hi]])."""
        row = np.asarray(row, np.uint64)
        lo = int(self.cuts[rank])
        a, b = int(self.ccuts[rank, c]), int(self.ccuts[rank, c + 1])
        base = int(row[lo])
        row_loc = (row[a:b + 1] - row[a]).astype(np.uint64)
        src = np.asarray(col_rows)[int(row[a]) - base:int(row[b]) - base]
        return row_loc, self.slots(src)
