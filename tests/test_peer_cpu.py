"""CPU: the peer-store exchange's address arithmetic.

The ranks' shared buffers are emulated as regions of one flat float32 "address space" at arbitrary
(256-byte aligned, unordered) base addresses.  Every output element of both layers is stored through
the view formula the kernels use (base + (a - row0)*s_row + tab[c / cblk] + (c % cblk)*s_col) with the
tables of peer_block_tables, and the receiving buffers must then hold exactly what the all-to-all
exchange delivers (blocks_to_cols / cols_to_blocks semantics)."""

import ctypes

import numpy as np
import pytest

from boltz_mlx_b200 import _lib
from boltz_mlx_b200.build import build
from boltz_mlx_b200.distributed import peer_block_tables, peer_layout

C = 128


def _space(N, P, seed):
    lay = peer_layout(N, P)
    rng = np.random.default_rng(seed)
    gap = (lay["total"] + 4095) // 4096 * 4096
    order = rng.permutation(P)  # buffers in a shuffled order, with gaps, some below the own one
    ptrs = [int(4096 + (order[q] * 2 + 1) * gap) for q in range(P)]
    mem = np.full((max(ptrs) + gap) // 4, np.nan, np.float32)
    return lay, ptrs, mem


@pytest.mark.parametrize("N,P", [(8, 1), (8, 2), (12, 3), (16, 4), (16, 8)])
def test_peer_tables_route_every_block(N, P):
    lay, ptrs, mem = _space(N, P, seed=N * 10 + P)
    R = N // P
    g = np.random.default_rng(1)
    y_start = g.standard_normal((N, N, C), dtype=np.float32)  # start output at (row i, col j)
    y_end = g.standard_normal((N, N, C), dtype=np.float32)    # end output at (row i, col j)
    ch = np.arange(C)
    for p in range(P):
        t_start, t_end, flags = peer_block_tables(ptrs, p, N, P)
        assert flags == [ptrs[q] + lay["flags"] for q in range(P)]
        r0 = p * R
        base = (ptrs[p] + lay["zc"]) // 4
        for a in range(r0, r0 + R):  # starting node: attention row a = row i, column c = j
            for c in range(N):
                off = base + (a - r0) * (R * C) + t_start[c // R] + (c % R) * C
                mem[off + ch] = y_start[a, c]
    for q in range(P):  # rank q's column buffer = the all-to-all's recv viewed as [N, R, C]
        zc = mem[(ptrs[q] + lay["zc"]) // 4:][:N * R * C].reshape(N, R, C)
        np.testing.assert_array_equal(zc, y_start[:, q * R:(q + 1) * R])
    for q in range(P):
        _, t_end, _ = peer_block_tables(ptrs, q, N, P)
        r0 = q * R
        base = (ptrs[q] + lay["zb"]) // 4
        for a in range(r0, r0 + R):  # ending node: attention row a = column j of z, c = row i
            for c in range(N):
                off = base + (a - r0) * C + t_end[c // R] + (c % R) * (R * C)
                mem[off + ch] = y_end[c, a]
    for p in range(P):  # rank p's row blocks: zb[q][i_l][j_l] = z[p R + i_l][q R + j_l]
        zb = mem[(ptrs[p] + lay["zb"]) // 4:][:P * R * R * C].reshape(P, R, R, C)
        want = y_end[p * R:(p + 1) * R].reshape(R, P, R, C).transpose(1, 0, 2, 3)
        np.testing.assert_array_equal(zb, want)


def test_peer_layout_keeps_regions_apart():
    for N, P in [(1024, 2), (1024, 8), (2048, 4), (768, 6)]:
        lay = peer_layout(N, P)
        R = N // P
        assert lay["zb"] - lay["zc"] == N * R * C * 4
        assert lay["flags"] - lay["zb"] == P * R * R * C * 4
        assert lay["ws"] - lay["flags"] >= 4 * P
        assert lay["zb"] % 256 == 0 and lay["flags"] % 256 == 0 and lay["ws"] % 256 == 0
        assert peer_layout(N, P, ws_bytes=1000)["total"] == lay["ws"] + 1000


def test_peer_tables_reject_misaligned_buffers():
    lay = peer_layout(8, 2)
    with pytest.raises(ValueError):
        peer_block_tables([4096, 4096 + lay["total"] + 2], 0, 8, 2)


def test_peer_entry_points_validate_on_the_host():
    build()
    L = _lib.lib()
    p = ctypes.c_void_p()
    assert L.triattn_peer_alloc(0, ctypes.byref(p)) == _lib.EINVAL
    assert L.triattn_peer_alloc(256, None) == _lib.EINVAL
    assert L.triattn_ipc_open(None, ctypes.byref(p)) == _lib.EINVAL
    assert L.triattn_ipc_handle(None, ctypes.create_string_buffer(64)) == _lib.EINVAL
    assert L.triattn_peer_free(None) == _lib.OK
    assert L.triattn_ipc_close(None) == _lib.OK
    # barrier: table, rank and world checked before any launch
    assert L.triattn_peer_barrier(None, 0, 2, 1, None) == _lib.EINVAL
    assert L.triattn_peer_barrier(4096 + 4, 0, 2, 1, None) == _lib.EINVAL
    assert L.triattn_peer_barrier(4096, 2, 2, 1, None) == _lib.EINVAL
    assert L.triattn_peer_barrier(4096, 0, 33, 1, None) == _lib.EINVAL
    # broadcast: table, rank and 16-byte granularity checked before any launch
    assert L.triattn_peer_broadcast(None, 0, 2, 0, 256, None) == _lib.EINVAL
    assert L.triattn_peer_broadcast(4096, 3, 2, 0, 256, None) == _lib.EINVAL
    assert L.triattn_peer_broadcast(4096, 0, 2, 8, 256, None) == _lib.EINVAL
    assert L.triattn_peer_broadcast(4096, 0, 2, 0, 250, None) == _lib.EINVAL
    # block-table output projection: the table is required and must be 8-byte aligned
    N, R = 256, 128
    args = dict(z=4096, out=8192, packed=256 * 64, ws=256 * 128)

    def vt(table, cblk=R):
        return L.triattn_out_proj_vt(args["z"], N * N * C, R * C, C, R, R * R * C, args["out"], N * R * C, R * C, C,
                                     cblk, table, args["packed"], 1, N, 0, R, _lib.BF16, 1, args["ws"], 1 << 34, None)

    assert vt(None) == _lib.EINVAL
    assert vt(4096 + 4) == _lib.EINVAL
    assert vt(4096, cblk=0) == _lib.EINVAL
    assert vt(4096, cblk=100) == _lib.EINVAL  # blocks must divide N
