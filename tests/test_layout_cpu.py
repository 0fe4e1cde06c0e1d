"""CPU emulation of the tensor-core operand addressing (in the spirit of the reference's
tests/nax3_emul.py): the byte layout the producers write must be exactly what the UMMA shared-memory
descriptors of the consumers read, for every MMA the kernels issue."""

import numpy as np
import pytest

from boltz_mlx_b200.layout import TILE, Workspace, bias16_offsets, img_offsets, sw128_offsets


def kmajor_desc_addr(start, lbo, sbo, rows, kdim):
    """Bytes read by a no-swizzle K-major descriptor for a rows x kdim (16-bit) operand."""
    r = np.arange(rows)[:, None]
    k = np.arange(kdim)[None, :]
    return start + (r % 8) * 16 + (r // 8) * sbo + (k % 8) * 2 + (k // 8) * lbo


def mnmajor_desc_addr(start, lbo, sbo, mn, kdim):
    """Bytes read by a no-swizzle MN-major descriptor: element (mn, k)."""
    m = np.arange(mn)[:, None]
    k = np.arange(kdim)[None, :]
    return start + (k % 8) * 16 + (k // 8) * lbo + (m % 8) * 2 + (m // 8) * sbo


def sw128_desc_addr(start, rows, kdim):
    """Bytes read by a 128-byte-swizzle K-major descriptor (SBO 1024) for rows x kdim 16-bit values:
    the unswizzled address start + (r // 8) * 1024 + (r % 8) * 128 + 2 k, then the hardware XORs
    address bits [4,7) with bits [7,10) (the start must keep the atom 1024-byte aligned)."""
    r = np.arange(rows)[:, None]
    k = np.arange(kdim)[None, :]
    a = start + (r // 8) * 1024 + (r % 8) * 128 + 2 * k
    return a ^ (((a >> 7) & 7) << 4)


@pytest.mark.parametrize("kdim", [32, 128])
def test_image_is_a_dense_bijection(kdim):
    off = img_offsets(TILE, kdim)
    assert off.min() == 0 and off.max() == TILE * kdim * 2 - 2
    assert len(np.unique(off)) == TILE * kdim
    assert np.all(off % 2 == 0)
    # every 8-row x 8-element core matrix is one contiguous 128-byte block
    for r0 in range(0, TILE, 8):
        for k0 in range(0, kdim, 8):
            blk = np.sort(off[r0:r0 + 8, k0:k0 + 8].ravel())
            assert blk[0] % 128 == 0 and np.array_equal(np.diff(blk), np.full(63, 2))


def test_qk_mma_k_steps():
    """S = Q K^T: two K=16 instructions at start + 256 B (lbo 128, sbo 512) cover the 32-channel image."""
    off = img_offsets(TILE, 32)
    for ks in range(2):
        got = kmajor_desc_addr(ks * 256, 128, 512, TILE, 16)
        assert np.array_equal(got, off[:, ks * 16:(ks + 1) * 16])


def test_pv_mma_reads_v_image_as_mn_major():
    """O = P V: B = V (N = 32 channels, K = 128 keys) MN-major with lbo 512 / sbo 128; instruction j
    (keys 16j..16j+15) starts at +1024 j.  The V image is written K-major by ln_proj (row = key)."""
    off = img_offsets(TILE, 32)  # off[key, ch]
    for j in range(TILE // 16):
        got = mnmajor_desc_addr(j * 1024, 512, 128, 32, 16)  # [ch, key-in-step]
        assert np.array_equal(got, off[j * 16:(j + 1) * 16, :].T)


@pytest.mark.parametrize("n_half", [0, 1])
def test_projection_mma_w_halves(n_half):
    """D[128 x 512] in two N=256 MMAs: B half h starts at +65536 B, K steps of 16 at +256 B."""
    woff = img_offsets(512, 128)
    aoff = sw128_offsets(TILE, 128)
    for ks in range(8):
        # A: swizzled LayerNorm image, K block ks // 4 at +16 KB, K step ks % 4 at +32 B inside an atom
        a = sw128_desc_addr((ks // 4) * TILE * 128 + (ks % 4) * 32, TILE, 16)
        assert np.array_equal(a, aoff[:, ks * 16:(ks + 1) * 16])
        b = kmajor_desc_addr(n_half * 65536 + ks * 256, 128, 2048, 256, 16)
        assert np.array_equal(b, woff[n_half * 256:(n_half + 1) * 256, ks * 16:(ks + 1) * 16])


def test_sw128_image_rows_are_two_contiguous_runs():
    """The swizzled image is a dense bijection, and one row's 128 channels are two 128-byte runs
    (a warp storing one row touches each shared-memory bank once per run)."""
    off = sw128_offsets(TILE, 128)
    assert len(np.unique(off)) == TILE * 128 and off.min() == 0 and off.max() == TILE * 256 - 2
    for r in range(TILE):
        for kb in range(2):
            run = np.sort(off[r, 64 * kb:64 * kb + 64])
            assert run[0] % 128 == 0 and np.array_equal(np.diff(run), np.full(63, 2))


def test_p_tmem_columns_pack_key_pairs():
    """P (128 queries x 128 keys, 16-bit) lives in TMEM columns [0,64): column c of lane q holds keys
    2c (low half) and 2c+1 (high half); TS instruction j reads columns 8j..8j+7 = keys 16j..16j+15."""
    cols = np.arange(64)
    keys_lo, keys_hi = 2 * cols, 2 * cols + 1
    for j in range(8):
        sel = slice(8 * j, 8 * j + 8)
        assert set(keys_lo[sel]) | set(keys_hi[sel]) == set(range(16 * j, 16 * j + 16))


@pytest.mark.parametrize("N", [1, 127, 128, 129, 1024, 2048])
def test_workspace_regions_disjoint_and_aligned(N):
    for dtype in (0, 1, 2):
        w = Workspace.make(2, N, N, dtype)
        offs = [w.off_bias, w.off_q, w.off_k, w.off_v, w.off_g, w.off_core, w.off_mb, w.total]
        assert offs == sorted(offs)
        assert all(o % 256 == 0 for o in offs)
        b0, b1 = w.bias_rows(0, N)
        assert b0 == w.off_bias == 0 and b1 <= w.off_q
        # the bias region does not move with the row count of a call
        for R in (1, max(1, N // 3), N):
            assert Workspace.make(2, N, R, dtype).off_bias == 0
            assert Workspace.make(2, N, R, dtype).off_q == w.off_q


def test_square_image_mma_k_steps():
    """The 128 x 128 MMAs (attention output projection, tri-mult tail: A = gated core / norm_out(o),
    B = W_o / p_out): K steps of 16 at +256 B with lbo 128 / sbo 2048 cover the whole K-major image."""
    off = img_offsets(TILE, 128)
    for ks in range(8):
        got = kmajor_desc_addr(ks * 256, 128, 16 * 128, TILE, 16)
        assert np.array_equal(got, off[:, ks * 16:(ks + 1) * 16])


@pytest.mark.parametrize("half", [0, 1])
def test_tri_bias_block_reads_as_a_kmajor_operand(half):
    """One 32 KB tri-bias block ([k/8][q][8] fp16, queries x keys) is a K-major operand with K core
    matrices 2048 B apart (lbo) and 8-query groups 128 B apart (sbo): K steps of 16 keys start every
    4096 B, so the keys 64 half .. 64 half + 63 of S are four steps from (8 half) x 2048."""
    N = 256
    NT = N // TILE
    full = bias16_offsets(N, 1, NT)[0, 0]  # [q, k] byte offsets, batch 0 head 0
    blk = full[:TILE, :TILE] - full[0, 0]  # block (qt 0, kt 0): offsets inside its 32 KB
    assert blk.min() == 0 and blk.max() == 32768 - 2
    for k4 in range(4):
        k0 = 64 * half + 16 * k4
        got = kmajor_desc_addr((8 * half + 2 * k4) * 2048, 2048, 128, TILE, 16)
        assert np.array_equal(got, blk[:, k0:k0 + 16])
