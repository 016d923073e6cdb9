"""Host-side arithmetic of the peer-memory reduce-scatter (no GPU): the byte layout of a rank's receive
buffer and the addresses each rank writes, for every world size the kernels accept (1-8) and the 8B /
70B shapes and decode-size slices.  The checks: regions of one buffer never overlap and stay inside it,
the two parities of a rank's slot and of its route rows are disjoint, the slots a rank writes into the
other ranks' buffers are exactly the ones the owner's combine reads (slot w at w * rows * D elements of
the parity's region), every address a TMA store or a 16-byte copy starts from is 16-byte aligned when the
row count divides by 4 (the peer path's precondition), and both flag arrays fit in the flag area."""

from __future__ import annotations

import itertools

import pytest

from conftest import fsi

sharding = fsi.sharding
PEER_FLAG_BYTES = fsi.kernels.PEER_FLAG_BYTES


def _regions(lay, world):
    regs = [("flags", 0, PEER_FLAG_BYTES)]
    for par, w in itertools.product(range(2), range(world)):
        regs.append((f"slot{par}.{w}", lay["slots"] + (par * world + w) * lay["slot"], lay["slot"]))
    for par in range(2):
        base = lay["routes"] + par * lay["route_par"]
        regs.append((f"ids{par}", base, lay["ids_bytes"]))
        regs.append((f"cnt{par}", base + lay["ids_bytes"], lay["route_par"] - lay["ids_bytes"]))
    return regs


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("M,D,cap,esize", [(16384, 4096, 56, 2), (16384, 8192, 112, 2), (16384, 4096, 56, 4),
                                           (2048, 4096, 8, 2), (512, 512, 5, 2)])
def test_peer_buffer_layout(world, M, D, cap, esize):
    rows = M // world
    lay = sharding.peer_layout(world, rows, D, esize, cap)
    regs = sorted(_regions(lay, world), key=lambda r: r[1])
    for (n0, a0, s0), (n1, a1, _) in zip(regs, regs[1:]):
        assert a0 + s0 <= a1, (n0, n1)  # disjoint, in address order
    assert regs[-1][1] + regs[-1][2] <= lay["total"]
    # flags: output flags at word w, route flags at byte 128 + 4 w, both inside the flag area
    assert 4 * 8 <= sharding.PeerReduce.ROUTE_FLAGS and sharding.PeerReduce.ROUTE_FLAGS + 4 * 8 <= PEER_FLAG_BYTES
    # what rank r writes on rank o (slot r of parity p) is slot r of the parity region the owner combines
    for r, p in itertools.product(range(world), range(2)):
        written = lay["slots"] + (p * world + r) * lay["slot"]
        combine_region = lay["slots"] + p * world * lay["slot"]
        assert written == combine_region + r * rows * D * esize
        assert written % 16 == 0
    # route rows of rank r: ids at r * rows * cap * 4, counts at r * rows * 4 into the parity's tables
    if rows % 4 == 0:
        for r, p in itertools.product(range(world), range(2)):
            ids = lay["routes"] + p * lay["route_par"] + r * rows * cap * 4
            cnt = lay["routes"] + p * lay["route_par"] + lay["ids_bytes"] + r * rows * 4
            assert ids % 16 == 0 and cnt % 16 == 0
            assert (rows * cap * 4) % 16 == 0 and (rows * 4) % 16 == 0  # whole 16-byte words per copy
            assert ids + rows * cap * 4 <= lay["routes"] + p * lay["route_par"] + lay["ids_bytes"]
            assert cnt + rows * 4 <= lay["routes"] + (p + 1) * lay["route_par"]
