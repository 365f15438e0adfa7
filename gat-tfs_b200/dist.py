"""Row-partitioned multi-GPU forward: one process per GPU, NCCL over NVLink.

Destination rows are cut into contiguous ranges balanced by edge count: rank k
owns rows [cuts[k], cuts[k+1]) with cuts[k] the first row whose CSR offset
reaches k*E/G. Destination rows are independent given the projected features
of all their sources, so each layer is

  1. projection of the rank's own rows (tcgen05 kernel): H_k, L_k, R_k;
  2. one all-gather of H (and of R) into every rank's feature table;
  3. edge-softmax aggregation of the rank's own rows from that table.

The all-gather is the only exchange. Two ways to do it:

  exchange="p2p" (default): the feature tables are device allocations every
    rank maps (CUDA IPC over NVLink). The projection kernel stores each H and R
    tile into the local table and into every peer's table itself
    (gat_b200_projection_scatter), so the exchange runs inside the projection,
    tile by tile; a cross-GPU flag barrier (gat_b200_peer_barrier) then orders
    those stores before any rank's aggregation.
  exchange="dma": the projection writes the local table only and the copy
    engines push each chunk's block to every peer (one cudaMemcpyAsync per
    peer on its own stream) while the next chunk is aggregated; the same
    barrier follows. The copies take no SMs, so with several chunks the
    exchange overlaps the aggregation.
  exchange="nccl": the projection writes a send block and NCCL's all-gather
    moves it; each chunk's all-gather runs on NCCL's stream while the next
    chunk is aggregated.

Under p2p and dma, layer 1 exchanges its BF16 input rows (din padded, 208 bytes
per row on c4) rather than H (512 bytes): the copy engines push each rank's
converted rows into every peer's input table and every rank then projects the
whole table itself, which costs less than moving H.

Rows of a rank may be cut into `chunks` row chunks (balanced by edges, each
with its own CSR slice and degree schedule): aggregating chunk c of layer l
yields the chunk's rows of layer l+1's input, which are projected (and
exchanged) at once. Each layer has its own table, so a layer's exchange never
overwrites rows that another layer's aggregation, on any rank, may still read:
a rank writes layer l's table of step s+1 only after the barrier of layer
l+1 of step s, which every rank reaches after its layer-l aggregation.

The feature table is chunk-major: ncclAllGather moves equal blocks, so chunk c
of every rank is padded to the largest chunk (chunk_max rows) and the table
holds, for c = 0..chunks-1, the chunk-c blocks of ranks 0..G-1 one after the
other. Source s, owned by rank r at local chunk c and offset i, sits at table
row (c*G + r)*chunk_max + i; every CSR slice's source ids are remapped to
those rows once.
"""
from __future__ import annotations

from typing import Optional, Sequence

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


class PartitionedModel:
    """Three-layer BF16 forward of this rank's rows (bench/main.cpp:171-172 per
    rank). Each layer's H and R reach every rank's table through peer stores
    from the projection kernel ("p2p"), copy-engine pushes ("dma") or NCCL
    all-gathers ("nccl"); under p2p and dma layer 1 moves its BF16 input rows
    instead of H when they are narrower."""

    def __init__(self, row: np.ndarray, col_rows: np.ndarray, params: Sequence[G.Param], rank: int, world: int,
                 stream=None, dist_module=None, cuts: Optional[np.ndarray] = None, chunks: int = 1,
                 exchange: str = "p2p"):
        """row: all n+1 row pointers; col_rows: the sources of this rank's rows
        (col[row[cuts[rank]]:row[cuts[rank+1]]]); cuts: partition(row, world)."""
        import torch
        if exchange not in ("p2p", "dma", "nccl"):
            raise ValueError("exchange must be 'p2p', 'dma' or 'nccl'")
        if exchange != "nccl" and world > 8:
            raise ValueError("peer-memory exchanges support up to 8 ranks (one NVLink node)")
        self.torch = torch
        self.dist = dist_module
        self.exchange = exchange
        self.rank, self.world = rank, world
        self.lay = Layout(row, world, chunks, cuts)
        self.cuts = self.lay.cuts
        lo, hi = int(self.cuts[rank]), int(self.cuts[rank + 1])
        if len(col_rows) != int(row[hi]) - int(row[lo]):
            raise ValueError("col_rows must hold the sources of the rank's rows")
        self.n_loc = hi - lo
        self.e_loc = len(col_rows)
        self.stream = stream
        self.chunks = []  # (first local row, end local row, DeviceGraph or None)
        for c in range(chunks):
            a, b = self.lay.chunk_rows(rank, c)
            g = None
            if b > a:
                rl, cl = self.lay.slice_chunk(row, col_rows, rank, c)
                g = G.DeviceGraph(rl, cl, stream, n_src=self.lay.n_table)
            self.chunks.append((a, b, g))
        self.layers = [G.DeviceLayer(p) for p in params]
        self.din = params[0].in_
        self.classes = params[2].width
        self.ldh = [G.padded_ld(p.width, G.BF16) for p in params]
        self.heads = [p.heads for p in params]
        dev = torch.device("cuda", torch.cuda.current_device())
        self.ld0 = G.padded_ld(self.din, G.BF16)
        self.ld_hidden = G.padded_ld(max(params[0].width, params[1].width), G.BF16)
        n, cm, P, nt = self.n_loc, self.lay.chunk_max, chunks, self.lay.n_table
        i16 = torch.int16
        self.x_f32 = torch.empty((n, self.din), dtype=torch.float32, device=dev)
        self.x0 = torch.zeros((n, self.ld0), dtype=i16, device=dev)
        self.left = [torch.zeros((n * 8,), dtype=torch.float32, device=dev) for _ in range(2)]
        self.xs = [torch.zeros((n, self.ld_hidden), dtype=i16, device=dev) for _ in range(2)]
        self.logits = torch.empty((n, self.classes), dtype=torch.float32, device=dev)
        self._owned, self._mapped = [], []
        self.x_exchange = False
        if exchange in ("p2p", "dma"):
            # h_tab[l][j] / r_tab[l][j]: device pointer of rank j's layer-l table in this process
            own, handles = [], []
            for l in range(3):
                for nbytes in (nt * self.ldh[l] * 2, nt * self.heads[l] * 4):
                    ptr, h = G.peer_alloc(nbytes)
                    self._owned.append(ptr)
                    own.append(ptr)
                    handles.append(h)
            fptr, fh = G.peer_alloc(64)
            self._owned.append(fptr)
            own.append(fptr)
            handles.append(fh)
            # layer 1 exchanges its BF16 input rows instead of H when they are narrower
            self.x_exchange = world > 1 and self.ld0 < self.ldh[0]
            if self.x_exchange:
                xptr, xh = G.peer_alloc(nt * self.ld0 * 2)
                self._owned.append(xptr)
                own.append(xptr)
                handles.append(xh)
            allh = self._all_gather_bytes(b"".join(handles), dev)
            hb = G.PEER_HANDLE_BYTES
            ptrs = []  # [rank][table]: H/R of layers 1-3, flags, (layer-1 input)
            for j in range(world):
                if j == rank:
                    ptrs.append(own)
                    continue
                row_ptrs = []
                for k in range(len(own)):
                    p_ = G.peer_open(allh[j][k * hb:(k + 1) * hb])
                    self._mapped.append(p_)
                    row_ptrs.append(p_)
                ptrs.append(row_ptrs)
            self.h_tab = [[ptrs[j][2 * l] for j in range(world)] for l in range(3)]
            self.r_tab = [[ptrs[j][2 * l + 1] for j in range(world)] for l in range(3)]
            self.flags = [ptrs[j][6] for j in range(world)]
            self.epoch = 0
            self.peers = [j for j in range(world) if j != rank]
            # one copy stream per peer (copy engines, no SMs): dma pushes and the
            # layer-1 input exchange
            need_copies = exchange == "dma" or self.x_exchange
            self.copy_streams = [torch.cuda.Stream(device=dev) for _ in self.peers] if need_copies else []
            if self.x_exchange:
                self.x_tab = [ptrs[j][7] for j in range(world)]
                self.left0 = torch.zeros((nt * self.heads[0],), dtype=torch.float32, device=dev)
        else:
            ldh_max = max(self.ldh)
            self.h_send = torch.zeros((P, cm * ldh_max), dtype=i16, device=dev)
            self.r_send = torch.zeros((P, cm * 8), dtype=torch.float32, device=dev)
            self.h_full = [torch.zeros((nt * self.ldh[l],), dtype=i16, device=dev) for l in range(3)]
            self.r_full = [torch.zeros((nt * self.heads[l],), dtype=torch.float32, device=dev) for l in range(3)]
        self.events = None
        self.pending = []
        self._pipe = None

    def _all_gather_bytes(self, blob: bytes, dev):
        """Every rank's `blob` (same length on all ranks), as a list of bytes."""
        torch = self.torch
        if self.world == 1:
            return [blob]
        t = torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(dev)
        out = torch.empty((self.world * len(blob),), dtype=torch.uint8, device=dev)
        self.dist.all_gather_into_tensor(out, t)
        a = out.cpu().numpy().reshape(self.world, len(blob))
        return [a[j].tobytes() for j in range(self.world)]

    def enable_timing(self, on: bool):
        torch = self.torch
        self.events = [torch.cuda.Event(enable_timing=True) for _ in range(7)] if on else None

    def _mark(self, i):
        # 0 start, 1 after the input copy, 2 after layer 1's projections,
        # 3+l once layer l's exchange is complete, 6 end
        if self.events is not None:
            self.events[i].record(self.torch.cuda.current_stream())

    def _project(self, l: int, c: int, x, ldx):
        """Projection of chunk c's rows for layer l and their exchange."""
        p = self.layers[l]
        a, b, _ = self.chunks[c]
        cm, W, K, ldh = self.lay.chunk_max, self.world, p.heads, self.ldh[l]
        left = self.left[l & 1][a * K:b * K]
        if self.exchange == "dma":
            if b <= a:
                return
            torch = self.torch
            row0 = (c * W + self.rank) * cm
            h_own = self.h_tab[l][self.rank] + row0 * ldh * 2
            r_own = self.r_tab[l][self.rank] + row0 * K * 4
            G.projection(p, b - a, x[a:b], ldx, G.BF16, h_own, G.BF16, ldh, left, r_own, self.stream)
            if self.peers:
                ev = torch.cuda.Event()
                ev.record(torch.cuda.current_stream())
                for cs in self.copy_streams:
                    cs.wait_event(ev)
                G.copy_to_peers(h_own, [self.h_tab[l][j] + row0 * ldh * 2 for j in self.peers], (b - a) * ldh * 2,
                                self.copy_streams)
                G.copy_to_peers(r_own, [self.r_tab[l][j] + row0 * K * 4 for j in self.peers], (b - a) * K * 4,
                                self.copy_streams)
            return
        if self.exchange == "p2p":
            if b <= a:
                return
            row0 = (c * W + self.rank) * cm  # first table row of this block
            hs = [self.h_tab[l][j] + row0 * ldh * 2 for j in range(W)]
            rs = [self.r_tab[l][j] + row0 * K * 4 for j in range(W)]
            peers = [j for j in range(W) if j != self.rank]
            G.projection_scatter(p, b - a, x[a:b], ldx, hs[self.rank], ldh, left, rs[self.rank],
                                 [hs[j] for j in peers], [rs[j] for j in peers], self.stream)
            return
        torch = self.torch
        hs = self.h_send[c, : cm * ldh]
        rs = self.r_send[c, : cm * K]
        if b > a:
            G.projection(p, b - a, x[a:b], ldx, G.BF16, hs, G.BF16, ldh, left, rs, self.stream)
        hf = self.h_full[l][c * W * cm * ldh:(c + 1) * W * cm * ldh]
        rf = self.r_full[l][c * W * cm * K:(c + 1) * W * cm * K]
        if W > 1:
            # the feature tables hold BF16 bit patterns in int16 storage; NCCL has no
            # 16-bit integer type, so the exchange goes through a bfloat16 view
            self.pending.append(self.dist.all_gather_into_tensor(hf.view(torch.bfloat16), hs.view(torch.bfloat16),
                                                                  async_op=True))
            self.pending.append(self.dist.all_gather_into_tensor(rf, rs, async_op=True))
        else:
            hf.copy_(hs)
            rf.copy_(rs)

    def _exchange_input(self, xin):
        """Layer 1 with the input exchanged: each rank converts its rows into its
        blocks of the BF16 input table, the copy engines push them to every
        peer, and after the barrier every rank projects the whole table itself
        (H, L and R of all rows, locally). Same kernels on the same inputs, so
        the tables equal those of the H exchange bit for bit."""
        torch = self.torch
        cm, W, ld0 = self.lay.chunk_max, self.world, self.ld0
        comp = torch.cuda.current_stream()
        for c, (a, b, _) in enumerate(self.chunks):
            if b <= a:
                continue
            row0 = (c * W + self.rank) * cm
            dst = self.x_tab[self.rank] + row0 * ld0 * 2
            G.convert(b - a, self.din, xin[a:b], self.din, dst, ld0, self.stream)
            ev = torch.cuda.Event()
            ev.record(comp)
            for cs in self.copy_streams:
                cs.wait_event(ev)
            G.copy_to_peers(dst, [self.x_tab[j] + row0 * ld0 * 2 for j in self.peers], (b - a) * ld0 * 2,
                            self.copy_streams)
        self._complete()
        p = self.layers[0]
        G.projection(p, self.lay.n_table, self.x_tab[self.rank], ld0, G.BF16, self.h_tab[0][self.rank], G.BF16,
                     self.ldh[0], self.left0, self.r_tab[0][self.rank], self.stream)

    def _left(self, l, c, a, b):
        """L rows of chunk c (local rows [a, b)) for layer l."""
        K = self.heads[l]
        if l == 0 and self.x_exchange:
            row0 = (c * self.world + self.rank) * self.lay.chunk_max
            return self.left0[row0 * K:(row0 + b - a) * K]
        return self.left[l & 1][a * K:b * K]

    def _complete(self):
        """Every rank's projections of the current layer are in this rank's table."""
        if self.exchange in ("p2p", "dma"):
            if self.world > 1:
                comp = self.torch.cuda.current_stream()
                for cs in self.copy_streams:  # dma: this rank's pushes have landed
                    ev = self.torch.cuda.Event()
                    ev.record(cs)
                    comp.wait_event(ev)
                self.epoch += 1
                G.peer_barrier(self.flags, self.rank, self.epoch, self.stream)
            return
        for w in self.pending:
            w.wait()  # the current stream waits for NCCL's
        self.pending = []

    def _tables(self, l):
        if self.exchange in ("p2p", "dma"):
            return self.h_tab[l][self.rank], self.r_tab[l][self.rank]
        return self.h_full[l], self.r_full[l]

    def forward(self, x, logits, x_on_host: bool, logits_on_host: bool):
        """x: this rank's FP32 input rows [n_loc, din]; logits: [n_loc, classes]."""
        n = self.n_loc
        self._mark(0)
        xin = x
        if x_on_host:
            self.x_f32.copy_(x, non_blocking=True)
            xin = self.x_f32
        self._mark(1)
        if self.x_exchange:
            self._exchange_input(xin)
        else:
            G.convert(n, self.din, xin, self.din, self.x0, self.ld0, self.stream)
            for c in range(len(self.chunks)):
                self._project(0, c, self.x0, self.ld0)
        self._mark(2)
        dst_logits = logits if not logits_on_host else self.logits
        for l, p in enumerate(self.layers):
            if not (l == 0 and self.x_exchange):  # layer 1's tables are local then
                self._complete()
            self._mark(3 + l)
            K, ldh, last = p.heads, self.ldh[l], l == 2
            hf, rf = self._tables(l)
            for c, (a, b, g) in enumerate(self.chunks):
                if g is not None:
                    left = self._left(l, c, a, b)
                    if last:
                        G.aggregate_fused(g, K, p.dim, hf, G.BF16, ldh, left, rf, False,
                                          dst_logits[a:b], G.F32, p.width, self.stream)
                    else:
                        G.aggregate_fused(g, K, p.dim, hf, G.BF16, ldh, left, rf, True,
                                          self.xs[l][a:b], G.BF16, self.ld_hidden, self.stream)
                if not last:
                    self._project(l + 1, c, self.xs[l], self.ld_hidden)
        self._mark(6)
        if logits_on_host:
            logits.copy_(self.logits, non_blocking=True)

    def forward_async(self, x_host, logits_host):
        """Host-to-host forward for a stream of requests (the multi-GPU
        counterpart of gat_b200_model_forward_async): uploads this rank's rows
        of x_host (pinned FP32 [n_loc, din]) on an upload stream, runs the
        forward on the current stream (which must be the model's stream) and
        downloads the logits into logits_host (pinned) on a download stream,
        returning at once. Two device slots let request k's download and
        request k+1's upload overlap the compute. Host buffers must stay
        untouched until join() has been waited on."""
        torch = self.torch
        if self._pipe is None:
            dev = self.x0.device
            self._pipe = {
                "x": [torch.empty((self.n_loc, self.din), dtype=torch.float32, device=dev) for _ in range(2)],
                "y": [torch.empty((self.n_loc, self.classes), dtype=torch.float32, device=dev) for _ in range(2)],
                "up": torch.cuda.Stream(device=dev), "down": torch.cuda.Stream(device=dev),
                "uploaded": [torch.cuda.Event() for _ in range(2)],
                "computed": [torch.cuda.Event() for _ in range(2)],
                "downloaded": [torch.cuda.Event() for _ in range(2)],
                "used": [False, False], "k": 0,
            }
        P = self._pipe
        s = P["k"] & 1
        comp = torch.cuda.current_stream()
        if P["used"][s]:
            # slot s still serves request k-2: its X is free once that compute is
            # done, its logits once their download is
            P["up"].wait_event(P["computed"][s])
            comp.wait_event(P["downloaded"][s])
        with torch.cuda.stream(P["up"]):
            P["x"][s].copy_(x_host, non_blocking=True)
            P["uploaded"][s].record(P["up"])
        comp.wait_event(P["uploaded"][s])
        self.forward(P["x"][s], P["y"][s], False, False)
        P["computed"][s].record(comp)
        P["down"].wait_event(P["computed"][s])
        with torch.cuda.stream(P["down"]):
            logits_host.copy_(P["y"][s], non_blocking=True)
            P["downloaded"][s].record(P["down"])
        P["used"][s] = True
        P["k"] += 1

    def join(self):
        """The current stream waits (on the device) for every submitted
        forward_async request, downloads included."""
        if self._pipe is None:
            return
        comp = self.torch.cuda.current_stream()
        for s in range(2):
            if self._pipe["used"][s]:
                comp.wait_event(self._pipe["downloaded"][s])

    def launches(self) -> int:
        """Kernels one forward launches: the input conversion, per layer and
        chunk a projection and an aggregation (+ the hub merge of split rows),
        and one barrier per layer under the p2p exchange."""
        live = [g for _, _, g in self.chunks if g is not None]
        hub = sum(1 for g in live if g.info()["n_hub"])
        barriers = 3 if self.exchange != "nccl" and self.world > 1 else 0
        if self.x_exchange:
            # per chunk: convert; one whole-table projection; aggregations of 3 layers
            # (+ hub merges) and projections of layers 2-3 per chunk
            return len(live) + 1 + 3 * (len(live) + hub) + 2 * len(live) + barriers
        return 1 + 3 * (2 * len(live) + hub) + barriers

    def stage_times(self) -> dict:
        """ms of the last forward: layer 1's projection, then per layer the time
        from the completion of its exchange to the next one's (its aggregation,
        the next layer's projections and whatever exchange was not overlapped)."""
        torch = self.torch
        torch.cuda.synchronize()
        ev = self.events
        out = {"projection_l1": ev[1].elapsed_time(ev[2]), "wait_l1": ev[2].elapsed_time(ev[3])}
        for l in range(3):
            out[f"layer{l + 1}"] = ev[3 + l].elapsed_time(ev[4 + l] if l < 2 else ev[6])
        return out

    def close(self):
        """Frees the device state. Under the p2p exchange every rank must call
        it: peers may still store into this rank's tables until all ranks have
        finished their last forward."""
        torch = self.torch
        torch.cuda.synchronize()
        if self._owned and self.world > 1 and self.dist is not None:
            self.dist.barrier()
            torch.cuda.synchronize()
        for p_ in self._mapped:
            G.peer_close(p_)
        for p_ in self._owned:
            G.peer_free(p_)
        self._mapped, self._owned = [], []
        for l in self.layers:
            l.close()
        for _, _, g in self.chunks:
            if g is not None:
                g.close()
