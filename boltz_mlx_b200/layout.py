"""Host-side mirror of libtriattn's memory layout (boltz_mlx_b200/csrc/triattn_internal.cuh).

* Operand images: a 128-position x kdim-channel 16-bit tile stored as 8-row x 16-byte core matrices
  (the sm_100a UMMA no-swizzle K-major layout):
      byte(row, k) = (row % 8) * 16 + (row // 8) * (16 * kdim) + (k % 8) * 2 + (k // 8) * 128
* Workspace regions for attention rows [row_begin, row_end) of a B x N layer; the tri-bias region is
  first, at offset 0, whatever the row count.

Used by the row-sharded multi-GPU driver (to address the tri-bias rows it exchanges) and by the
stage-level tests (to decode operand images).  `workspace_bytes` must agree with the library's
triattn_workspace_bytes (checked by the CPU test-suite).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

TILE = 128
HEADS, C_HEAD, C_IN = 4, 32, 128
F32, F16, BF16 = 0, 1, 2


def align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


def round_tile(n: int) -> int:
    return (n + TILE - 1) // TILE * TILE


def img_offsets(rows: int, kdim: int) -> np.ndarray:
    """Byte offset of (row, k) inside an operand image, shape [rows, kdim]."""
    r = np.arange(rows)[:, None]
    k = np.arange(kdim)[None, :]
    return (r % 8) * 16 + (r // 8) * (16 * kdim) + (k % 8) * 2 + (k // 8) * 128


def sw128_offsets(rows: int, kdim: int) -> np.ndarray:
    """Byte offset of (row, k) in a 128-byte swizzled K-major image (the LayerNorm operand of the
    projection MMA): 64-element K blocks of rows * 128 bytes, 8-row atoms of 1024 bytes, the 16-byte
    chunk index XORed with row % 8.  Shape [rows, kdim]."""
    r = np.arange(rows)[:, None]
    k = np.arange(kdim)[None, :]
    return (r // 8) * 1024 + (r % 8) * 128 + ((((k % 64) // 8) ^ (r % 8)) * 16) + (k % 8) * 2 + (k // 64) * rows * 128


@dataclass
class Workspace:
    B: int
    N: int
    R: int
    dtype: int
    Np: int = 0
    NT: int = 0
    NTs: int = 0  # tile-class row stride: NT rounded up to 4
    off_q: int = 0
    off_k: int = 0
    off_v: int = 0
    off_g: int = 0
    off_core: int = 0
    off_bias: int = 0
    off_mb: int = 0
    off_ts: int = 0
    total: int = 0

    @classmethod
    def make(cls, B: int, N: int, R: int, dtype: int) -> "Workspace":
        w = cls(B, N, R, dtype)
        w.Np = round_tile(N)
        w.NT = w.Np // TILE
        w.NTs = (w.NT + 3) // 4 * 4
        o = 0
        # tri bias first: one fixed place for every row count (row chunks / ranks share it)
        w.off_bias = o
        o = align(o + (N * B * HEADS * w.Np * 4 if dtype == F32 else w.Np * B * HEADS * w.Np * 2))
        if dtype == F32:
            plane = B * R * N * C_IN * 4
            w.off_q = o; o = align(o + plane)
            w.off_k = o; o = align(o + plane)
            w.off_v = o; o = align(o + plane)
            w.off_g = o; o = align(o + plane)
            w.off_core = o; o = align(o + plane)
        else:
            head_tiles = B * R * HEADS * w.NT * 8192
            w.off_q = o; o = align(o + head_tiles)
            w.off_k = o; o = align(o + head_tiles)
            w.off_v = o; o = align(o + head_tiles)
            w.off_g = o; o = align(o + B * R * N * C_IN * 2)
            w.off_core = o; o = align(o + B * R * w.NT * 32768)
        w.off_mb = o; o = align(o + B * R * w.Np * 4)
        w.off_ts = o; o = align(o + B * R * w.NTs)
        w.total = o
        return w

    # byte range of the tri-bias rows [r0, r1): contiguous per row block.  fp32 path: layout
    # [N][B][H][Np] fp32.  16-bit path: 128-row blocks [qt][b][h][kt] (fp16), so r0 and r1 must be
    # multiples of 128 (or r1 = N for the last block).
    def bias_rows(self, r0: int, r1: int) -> tuple[int, int]:
        if self.dtype == F32:
            row = self.B * HEADS * self.Np * 4
            return self.off_bias + r0 * row, self.off_bias + r1 * row
        if r0 % TILE or (r1 % TILE and r1 != self.N):
            raise ValueError(f"16-bit tri-bias rows move in blocks of {TILE} rows: [{r0}, {r1})")
        row = self.B * HEADS * self.Np * 2
        return self.off_bias + r0 * row, self.off_bias + round_tile(r1) * row


def workspace_bytes(B: int, N: int, rows: int, dtype: int) -> int:
    return Workspace.make(B, N, rows, dtype).total


def bias16_offsets(N: int, B: int, NT: int):
    """Byte offsets [B, H, N(q), N(k)] of the 16-bit tri-bias blocks."""
    q = np.arange(N)[:, None]
    k = np.arange(N)[None, :]
    out = np.empty((B, HEADS, N, N), np.int64)
    for b in range(B):
        for h in range(HEADS):
            blk = (((q >> 7) * B + b) * HEADS + h) * NT + (k >> 7)
            out[b, h] = blk * 32768 + ((k & 127) >> 3) * 2048 + (q & 127) * 16 + (k & 7) * 2
    return out


def vimg_offsets() -> np.ndarray:
    """Byte offset of (key, ch) inside a 128 x 32 fp16 V image (MN-major), shape [128, 32]."""
    key = np.arange(TILE)[:, None]
    ch = np.arange(C_HEAD)[None, :]
    return (ch >> 3) * 2048 + (key >> 3) * 128 + (key & 7) * 16 + (ch & 7) * 2


def decode_v_images(buf, w: "Workspace"):
    """v images -> tensor [B, R, H, Np, 32] (fp16 values as float32)."""
    import torch

    n = w.B * w.R * HEADS * w.NT * 8192
    raw = buf[w.off_v:w.off_v + n].view(torch.float16).view(w.B, w.R, HEADS, w.NT, 4096)
    idx = torch.from_numpy(vimg_offsets() // 2).to(buf.device)
    return raw[..., idx].float().reshape(w.B, w.R, HEADS, w.Np, C_HEAD)


def decode_bias16(buf, w: "Workspace"):
    """16-bit tri bias -> tensor [B, H, N(q), N(k)] (log2 domain, float32)."""
    import torch

    n = w.Np * w.B * HEADS * w.Np * 2
    raw = buf[w.off_bias:w.off_bias + n].view(torch.float16)
    idx = torch.from_numpy(bias16_offsets(w.N, w.B, w.NT) // 2).to(buf.device)
    return raw[idx].float()


def decode_head_images(buf, w: Workspace, off: int):
    """q/k/v images -> tensor [B, R, H, Np, 32] (16-bit values as float32).  `buf` is a uint8 torch tensor."""
    import torch

    tdt = torch.bfloat16 if w.dtype == BF16 else torch.float16
    n = w.B * w.R * HEADS * w.NT * 8192
    raw = buf[off:off + n].view(tdt).view(w.B, w.R, HEADS, w.NT, 4096)
    idx = torch.from_numpy(img_offsets(TILE, C_HEAD) // 2).to(buf.device)
    return raw[..., idx].float().reshape(w.B, w.R, HEADS, w.Np, C_HEAD)


def decode_core_images(buf, w: Workspace):
    """core images (fp16 o / l, before the sigmoid gate, for both 16-bit precisions) -> tensor [B, R, Np, 128]."""
    import torch

    n = w.B * w.R * w.NT * 32768
    raw = buf[w.off_core:w.off_core + n].view(torch.float16).view(w.B, w.R, w.NT, 16384)
    idx = torch.from_numpy(img_offsets(TILE, C_IN) // 2).to(buf.device)
    return raw[..., idx].float().reshape(w.B, w.R, w.Np, C_IN)


# ---- triangle multiplication (csrc/triattn_internal.cuh: TrimulPacked, TrimulWorkspace) -------------
TM_D, TM_W1 = 128, 640
TRIMUL_BLAS_BYTES = 32 << 20


def trimul_packed_bytes(dtype: int) -> int:
    """Packed tri-mult weights: fp32 LayerNorm vectors (2 KB), W1 = p_in | g_in | g_out [640][128] and
    p_out [128][128] in fp32; 16-bit modes add both row-major in the layer's type, then the p_in | g_in
    (512 x 128) and p_out (128 x 128) operand images (1024-byte aligned)."""
    f32_end = 2048 + TM_W1 * TM_D * 4 + TM_D * TM_D * 4
    if dtype == F32:
        return align(f32_end)
    w1_16 = align(f32_end)
    p_out_16 = w1_16 + TM_W1 * TM_D * 2
    img_pg = align(p_out_16 + TM_D * TM_D * 2, 1024)
    img_po = img_pg + 5 * TM_D * TM_D * 2  # p_a | g_a | p_b | g_b | g_out image
    return align(img_po + TM_D * TM_D * 2)


def trimul_workspace_bytes(B: int, N: int, dtype: int) -> int:
    """Tri-mult workspace.  Channel planes of a, b and o are N rows of Np elements (16-bit: Np = N rounded
    up to 8, 16-byte aligned rows for the contraction's TMA loads; fp32: Np = N).
    fp32: xn [P][128], h [P][640], a|b (or p_out's fp32 output, whichever is larger), o, 32 MiB cuBLAS
    scratch.  16-bit: g_out [P][128], a|b [2][B][128][N][Np], o fp32 [B][128][N][Np]."""
    f32 = dtype == F32
    Np = N if f32 else (N + 7) // 8 * 8
    P, Pp = B * N * N, B * N * Np
    es = 4 if f32 else 2
    o = align(P * TM_D * es if f32 else 0)
    o = align(o + P * (TM_W1 if f32 else TM_D) * es)
    o = align(o + max(2 * Pp * TM_D * es, P * TM_D * 4 if f32 else 0))
    o = align(o + Pp * TM_D * 4)
    return align(o + (TRIMUL_BLAS_BYTES if f32 else 0))
