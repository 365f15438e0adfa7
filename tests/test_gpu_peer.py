"""Peer-memory exchange primitives on one GPU.

* gat_b200_projection_scatter: the "peer" destinations are further
  gat_b200_peer_alloc allocations on the same GPU, so the kernel's extra stores
  run without a second GPU; every destination must hold the local H and R bit
  for bit, including unaligned R blocks (heads = 1) and a ragged last tile.
* gat_b200_peer_barrier: a rank whose peer never arrives (a flag nothing sets)
  gives up after its bounded wait and the host reads GAT_B200_ETIMEOUT; the
  device stays usable. No kernel that waits on another launch runs on this GPU.
"""
import numpy as np
import pytest

import gatb200 as G

from test_gpu_parity import dev_bf16, random_layer

pytestmark = pytest.mark.gpu


class _Raw:
    """A raw device allocation seen as a 1-D array (CUDA array interface)."""

    def __init__(self, ptr, count, typestr):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3}


def _read(ptr, count, dtype):
    import torch
    torch.cuda.synchronize()
    G.check_device()
    typestr = {torch.int16: "<i2", torch.float32: "<f4", torch.int32: "<i4"}[dtype]
    a = torch.as_tensor(_Raw(ptr, count, typestr), device="cuda").cpu().numpy()
    return a.view(np.uint16) if a.dtype == np.int16 else a


@pytest.mark.parametrize("n,D,K,d,row0", [(1000, 100, 8, 32, 0), (333, 256, 8, 32, 4), (517, 256, 1, 47, 3)])
def test_projection_scatter_matches_local(dev, n, D, K, d, row0):
    import torch
    rng = np.random.default_rng(n + K)
    p = random_layer(rng, D, K, d)
    layer = G.DeviceLayer(p)
    ldx, W = G.padded_ld(D, G.BF16), K * d
    ldh = G.padded_ld(W, G.BF16)
    xb = dev_bf16(rng.standard_normal((n, D)).astype(np.float32), ldx)
    rows = n + row0 + 5
    allocs = [G.peer_alloc(rows * ldh * 2)[0] for _ in range(3)] + [G.peer_alloc(rows * K * 4)[0] for _ in range(3)]
    try:
        hs = [a + row0 * ldh * 2 for a in allocs[:3]]
        rs = [a + row0 * K * 4 for a in allocs[3:]]
        left = torch.empty((n, K), dtype=torch.float32, device="cuda")
        G.projection_scatter(layer, n, xb, ldx, hs[0], ldh, left, rs[0], hs[1:], rs[1:])
        # the plain projection as the reference for every copy
        h_ref = torch.zeros((n, ldh), dtype=torch.int16, device="cuda")
        r_ref = torch.empty((n, K), dtype=torch.float32, device="cuda")
        l_ref = torch.empty((n, K), dtype=torch.float32, device="cuda")
        G.projection(layer, n, xb, ldx, G.BF16, h_ref, G.BF16, ldh, l_ref, r_ref)
        torch.cuda.synchronize()
        want_h = h_ref.cpu().numpy().view(np.uint16)
        want_r = r_ref.cpu().numpy()
        assert np.array_equal(left.cpu().numpy(), l_ref.cpu().numpy())
        for k in range(3):
            got_h = _read(allocs[k], rows * ldh, torch.int16).reshape(rows, ldh)
            got_r = _read(allocs[3 + k], rows * K, torch.float32).reshape(rows, K)
            assert np.array_equal(got_h[row0:row0 + n], want_h), k
            assert np.array_equal(got_r[row0:row0 + n], want_r), k
            # rows outside the block stay untouched (zero-filled allocation)
            assert not got_h[:row0].any() and not got_h[row0 + n:].any()
            assert not got_r[:row0].any() and not got_r[row0 + n:].any()
    finally:
        for a in allocs:
            G.peer_free(a)
        layer.close()


def test_projection_scatter_rejects_bad_arguments(dev):
    import torch
    rng = np.random.default_rng(3)
    p = random_layer(rng, 64, 8, 32)
    layer = G.DeviceLayer(p)
    ldx, ldh = G.padded_ld(64, G.BF16), 256
    xb = dev_bf16(rng.standard_normal((10, 64)).astype(np.float32), ldx)
    h = torch.zeros((10, ldh), dtype=torch.int16, device="cuda")
    r = torch.zeros((10, 8), dtype=torch.float32, device="cuda")
    with pytest.raises(G.GatError, match="npeer"):
        G.projection_scatter(layer, 10, xb, ldx, h, ldh, None, r, [h.data_ptr()] * 8, [r.data_ptr()] * 8)
    with pytest.raises(G.GatError, match="16-byte"):
        G.projection_scatter(layer, 10, xb, ldx, h, ldh, None, r, [h.data_ptr() + 2], [r.data_ptr()])
    layer.close()


def test_peer_barrier_times_out_when_peer_never_arrives(dev):
    import time
    import torch
    own, _ = G.peer_alloc(64)
    other, _ = G.peer_alloc(64)  # stands in for rank 1's flags; nothing ever sets ours
    try:
        t0 = time.time()
        G.peer_barrier([own, other], 0, 1)
        torch.cuda.synchronize()
        with pytest.raises(G.GatError) as e:
            G.check_device()
        assert e.value.code == 4  # GAT_B200_ETIMEOUT
        assert time.time() - t0 < 30
        # the release went to the peer's slot of rank 0
        assert _read(other, 2, torch.int32)[0] == 1
        # the context is still usable and the error was cleared
        G.check_device()
        x = torch.ones(4, device="cuda") * 2
        assert float(x.sum()) == 8.0
    finally:
        G.peer_free(own)
        G.peer_free(other)


def test_peer_barrier_argument_checks(dev):
    with pytest.raises(G.GatError, match="world"):
        G.peer_barrier([0] * 9, 0, 1)
    with pytest.raises(G.GatError, match="rank"):
        G.peer_barrier([1, 2], 2, 1)
    G.peer_barrier([1], 0, 1)  # one rank: nothing to wait for, no launch
