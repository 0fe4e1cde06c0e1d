"""Row-sharded triangle attention over the GPUs of one node (one process per GPU, NCCL over NVLink).

The reference runs on one device and bounds memory by row chunking: the tri bias is computed from
ALL rows, then attention runs over chunks of rows (attention.py:55-68, kernels.py:1158-1168).  The
multi-GPU form distributes those row chunks:

* z (and the residual stream) is sharded by rows i: rank p owns rows [p*R, (p+1)*R), R = N / P.
* Starting node: LN + projection of the local rows, their tri-bias rows, ONE all-gather of the tri
  bias ([N][B][H][Np] fp32, rows contiguous), local attention core and output projection + residual.
* Ending node: attention row a is column a of z, so the pair tensor is re-sharded by columns with
  an all-to-all, the same stages run on the column block through strided views (no transposed copy
  of z is materialised by the kernels), the tri bias is all-gathered, and the updated column block
  goes back to row sharding with a second all-to-all.
* Block layout of the residual stream: a rank keeps its rows of z as [P][R][R][C] blocks (block p =
  the columns of rank p).  The starting node runs on it through a column-blocked view; block p is
  exactly the chunk all_to_all_single sends to rank p, and the ending node's column block, sent
  back, lands in the same layout.  So a start+end pair (pair_blocks) costs two all-to-alls and no
  transposing copy.  pair() wraps it for callers that hold row-layout shards [R][N][C].

Two exchanges move the blocks:

* exchange="nccl": the steps above as torch.distributed collectives (all_to_all_single), so the
  host logic also runs on CPU ranks with the gloo backend (tests/test_distributed_cpu.py).
* exchange="peer": no all-to-all at all.  Every rank's column buffer zc [N][R][C] and row-block
  buffer zb [P][R][R][C] live in one CUDA-IPC-shared allocation mapped on every rank.  The starting
  node's output projection reads z from zb and stores each output block straight into the column
  buffer of the rank that owns those columns (NVLink stores, overlapped with the projection); the
  ending node reads zc and stores its output blocks straight into the owners' zb.  A cross-GPU
  barrier (bounded flag waits, libtriattn's triattn_peer_barrier) after each output projection
  orders the layers.  The per-block destinations are a device table of element offsets
  (peer_block_tables).  The workspaces live in the shared allocation too: each rank stores its
  tri-bias rows into every other rank's bias region with one broadcast launch
  (triattn_peer_broadcast) and a barrier, in place of the all-gather.  The arithmetic per row is
  the same, so both exchanges give identical bits.
"""

from __future__ import annotations

import ctypes
import json
import os
from pathlib import Path
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib
from .layout import C_IN, Workspace


def shard_rows(N: int, P: int, rank: int) -> tuple[int, int]:
    if N % P:
        raise _lib.TriAttnUnsupported(_lib.EUNSUPPORTED, f"N={N} must be divisible by the {P} ranks")
    R = N // P
    return rank * R, (rank + 1) * R


def gather_bias(ws: torch.Tensor, w: Workspace, r0: int, r1: int, group=None) -> None:
    """All-gather the tri-bias rows [r0, r1) of every rank into the full bias region (in place)."""
    b0, b1 = w.bias_rows(0, w.N)
    full = ws[b0:b1]
    l0, l1 = w.bias_rows(r0, r1)
    local = ws[l0:l1]
    dist.all_gather_into_tensor(full, local.clone() if not full.is_cuda else local, group=group)


def rows_to_cols(z_loc: torch.Tensor, P: int, send: torch.Tensor, recv: torch.Tensor, group=None) -> torch.Tensor:
    """Row shard z_loc [R, N, C] -> column block zt [N, R, C] (zt[i, a] = z[i, r0 + a]) by all-to-all.

    send / recv are [P, R, R, C] buffers; the result is `recv` viewed as [N, R, C]."""
    R, N, Cc = z_loc.shape
    send.copy_(z_loc.view(R, P, R, Cc).transpose(0, 1))
    dist.all_to_all_single(recv, send, group=group)
    return recv.view(N, R, Cc)


def cols_to_rows(zt: torch.Tensor, P: int, recv: torch.Tensor, z_loc_out: torch.Tensor, group=None) -> None:
    """Column block zt [N, R, C] -> row shard z_loc_out [R, N, C] by all-to-all (inverse of rows_to_cols)."""
    N, R, Cc = zt.shape
    dist.all_to_all_single(recv, zt.reshape(P, R, R, Cc).contiguous(), group=group)
    z_loc_out.view(R, P, R, Cc).copy_(recv.transpose(0, 1))


def to_blocks(z_loc: torch.Tensor, P: int, z_blk: torch.Tensor) -> torch.Tensor:
    """Row shard [R, N, C] -> block layout [P, R, R, C] (z_blk[p, i, a] = z_loc[i, p*R + a])."""
    R, N, Cc = z_loc.shape
    z_blk.copy_(z_loc.view(R, P, R, Cc).transpose(0, 1))
    return z_blk


def from_blocks(z_blk: torch.Tensor, z_loc: torch.Tensor) -> torch.Tensor:
    """Block layout [P, R, R, C] -> row shard [R, N, C] (inverse of to_blocks)."""
    P, R, _, Cc = z_blk.shape
    z_loc.view(R, P, R, Cc).copy_(z_blk.transpose(0, 1))
    return z_loc


def blocks_to_cols(z_blk: torch.Tensor, recv: torch.Tensor, group=None) -> torch.Tensor:
    """Block layout [P, R, R, C] of my rows -> column block [N, R, C] of my columns (all-to-all:
    block p goes to rank p as-is).  recv is a [P, R, R, C] buffer; returns it viewed as [N, R, C]."""
    P, R, _, Cc = z_blk.shape
    dist.all_to_all_single(recv, z_blk, group=group)
    return recv.view(P * R, R, Cc)


def cols_to_blocks(zt: torch.Tensor, z_blk: torch.Tensor, group=None) -> None:
    """Column block [N, R, C] -> block layout [P, R, R, C] of my rows (all-to-all; rows p*R.. of zt
    go to rank p, which receives them as its block of my columns)."""
    P, R, _, Cc = z_blk.shape
    dist.all_to_all_single(z_blk, zt.view(P, R, R, Cc), group=group)


def all_ranks_ok(ok: bool, group=None, device: Optional[torch.device] = None) -> bool:
    """True on every rank iff `ok` is True on every rank of the group (one all-reduce, MIN): a setup
    step that can fail on some ranks only is then accepted or rejected by all of them together."""
    dev = device if device is not None and dist.get_backend(group) == "nccl" else torch.device("cpu")
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(int(t.item()))


def exchange_intact(sent_blk: torch.Tensor, recv_blk: torch.Tensor, group=None) -> bool:
    """Integrity check of a block all-to-all (blocks_to_cols / cols_to_blocks): block q of `sent_blk`
    went to rank q, block p of `recv_blk` came from rank p.  Every rank sends the float64 sum of each
    block it sent to the block's receiver, which compares it with the sum of what arrived.  True on
    every rank iff every block arrived intact on every rank (one small all-to-all + one vote).

    A diagnostic of the NCCL exchange, not run on the hot path (it costs a pass over the blocks and a
    host sync): call it after an exchange when verifying a deployment.  A block whose sum is inf or NaN
    on both sides (non-finite data sent intact) counts as intact."""
    P = sent_blk.shape[0]
    sent = sent_blk.reshape(P, -1).double().sum(1)
    got = torch.empty_like(sent)
    dist.all_to_all_single(got, sent.contiguous(), group=group)
    arrived = recv_blk.reshape(P, -1).double().sum(1)
    tol = 1e-9 * (arrived.abs().nan_to_num(posinf=0.0) + 1.0)
    close = (got - arrived).abs() <= tol
    same_nonfinite = (~torch.isfinite(got)) & (~torch.isfinite(arrived)) & (
        (got.isnan() & arrived.isnan()) | (got == arrived))
    ok = bool((close | same_nonfinite).all())
    return all_ranks_ok(ok, group, sent_blk.device)


class PeerUnavailable(RuntimeError):
    """Some rank could not map another rank's buffer (no peer access between those GPUs)."""


class _DeviceArray:
    """A raw device allocation described by __cuda_array_interface__ (torch.as_tensor wraps it
    without a copy; the wrapper keeps `owner` alive)."""

    def __init__(self, ptr: int, shape, typestr: str, owner):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}
        self._owner = owner


class PeerSpace:
    """One IPC-shared device buffer per rank (triattn_peer_alloc), mapped on every rank of the group:
    ptrs[q] is rank q's buffer as seen from this process (ptrs[rank] = the own buffer)."""

    def __init__(self, nbytes: int, device: torch.device, group=None):
        with torch.cuda.device(device):  # the allocation, the IPC mappings and the all-gather on `device`
            self._setup(nbytes, device, group)

    def _setup(self, nbytes: int, device: torch.device, group) -> None:
        L = _lib.lib()
        self.group, self.device, self.nbytes = group, device, nbytes
        self.P, self.rank = dist.get_world_size(group), dist.get_rank(group)
        own = ctypes.c_void_p()
        _lib.check(L.triattn_peer_alloc(nbytes, ctypes.byref(own)))
        self.own = own.value
        h = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        _lib.check(L.triattn_ipc_handle(self.own, h))
        handles = [None] * self.P
        dist.all_gather_object(handles, h.raw, group=group)
        self.ptrs, self._opened = [], []
        err = None
        for q, hq in enumerate(handles):
            if q == self.rank:
                self.ptrs.append(self.own)
                continue
            p = ctypes.c_void_p()
            rc = L.triattn_ipc_open(ctypes.create_string_buffer(hq, _lib.IPC_HANDLE_BYTES), ctypes.byref(p))
            if rc != _lib.OK:
                err = f"rank {self.rank} cannot map rank {q}'s buffer: {(L.triattn_last_error_string() or b'').decode()}"
                break
            self.ptrs.append(p.value)
            self._opened.append(p.value)
        if not all_ranks_ok(err is None, group, device):
            self.close()  # every rank unmaps what it mapped and frees its own buffer
            raise PeerUnavailable(err or "another rank could not map a peer buffer")

    def tensor(self, offset: int, shape, dtype=torch.float32) -> torch.Tensor:
        """A view of this rank's own buffer at byte `offset`."""
        typestr = {torch.float32: "<f4", torch.int64: "<i8", torch.int32: "<i4", torch.uint8: "|u1"}[dtype]
        n = 1
        for d in shape:
            n *= d
        if offset < 0 or offset + n * torch.empty((), dtype=dtype).element_size() > self.nbytes:
            raise ValueError(f"view [{offset}, +{shape}) outside the {self.nbytes}-byte peer buffer")
        return torch.as_tensor(_DeviceArray(self.own + offset, shape, typestr, self), device=self.device)

    def close(self) -> None:
        """Unmap the peers' buffers, then free the own one once every rank has unmapped it.  Call
        after the GPU work that uses them has finished, on every rank."""
        if self.own is None:
            return
        L = _lib.lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            for p in self._opened:
                _lib.check(L.triattn_ipc_close(p))
            self._opened = []
            dist.barrier(group=self.group)
            _lib.check(L.triattn_peer_free(self.own))
        self.own = None


def peer_layout(N: int, P: int, ws_bytes: int = 0) -> dict:
    """Byte offsets inside every rank's shared buffer: zc [N][R][C] fp32 (the rank's column block),
    zb [P][R][R][C] fp32 (the rank's rows in column blocks), flags [P] uint32 (barrier slots), ws
    (the rank's libtriattn workspace: peers store their tri-bias rows into its bias region)."""
    R = N // P
    zc = N * R * C_IN * 4
    ws = 2 * zc + (4 * P + 255) // 256 * 256
    return {"zc": 0, "zb": zc, "flags": 2 * zc, "ws": ws, "total": ws + ws_bytes}


def peer_block_tables(ptrs: list, rank: int, N: int, P: int) -> tuple[list, list, list]:
    """Destination tables of the peer exchange, element offsets for triattn_out_proj_vt.

    start: the starting node's output view (attention row a = row i of z, column c = j) has base =
      this rank's zc, s_row = R*C, s_col = C, blocks of R columns; block q lands in rank q's zc at
      [a][c % R] (zc_q + (a*R + c%R)*C), so tab[q] = (zc_q - zc_own)/4 + r0*R*C.
    end: the ending node's output view (a = column j of z, c = row i) has base = this rank's zb,
      s_row = C, s_col = R*C; block q lands in rank q's zb at [rank][c % R][a - r0], so
      tab[q] = (zb_q - zb_own)/4 + rank*R*R*C.
    flags: the address of every rank's barrier slots."""
    R, r0 = N // P, rank * (N // P)
    lay = peer_layout(N, P)

    def el(delta: int) -> int:
        if delta % 4:
            raise ValueError("peer buffers must be 4-byte aligned relative to one another")
        return delta // 4

    start = [el(ptrs[q] + lay["zc"] - (ptrs[rank] + lay["zc"])) + r0 * R * C_IN for q in range(P)]
    end = [el(ptrs[q] + lay["zb"] - (ptrs[rank] + lay["zb"])) + rank * R * R * C_IN for q in range(P)]
    flags = [ptrs[q] + lay["flags"] for q in range(P)]
    return start, end, flags


class ShardedPair:
    """One start+end triangle-attention pair on a row-sharded pair tensor (B = 1)."""

    def __init__(self, N: int, precision: str, device: torch.device, group=None, inf: float = 1e9,
                 exchange: str = "nccl", checked: bool = True):
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"exchange must be 'nccl' or 'peer', not {exchange!r}")
        self.N, self.inf, self.device, self.group, self.exchange = N, inf, device, group, exchange
        # checked: read the device status word after every pair (one host sync) and raise on any
        # error, so a bounded wait that ran out (a peer that never arrived, a stale error) is reported
        # instead of returning blocks whose exchange may have raced.  Timing loops may turn it off and
        # read the status once at the end.
        self.checked = checked
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.r0, self.r1 = shard_rows(N, self.P, self.rank)
        self.R = self.r1 - self.r0
        self.dt = _lib.dtype_code(precision)
        if self.dt != _lib.F32 and self.R % 128:
            raise _lib.TriAttnUnsupported(_lib.EUNSUPPORTED,
                                          f"16-bit row sharding needs rows per rank ({self.R}) to be a multiple of 128")
        self.w = Workspace.make(1, N, self.R, self.dt)
        self.L = _lib.lib()
        self.peer = None
        if exchange == "peer":
            self.lay = lay = peer_layout(N, self.P, self.w.total)
            try:
                self.peer = PeerSpace(lay["total"], device, group)
            except PeerUnavailable as e:  # all ranks together: the all-to-all exchange instead
                print(f"ShardedPair: peer exchange unavailable ({e}); using NCCL all-to-alls", flush=True)
                exchange = self.exchange = "nccl"
        if exchange == "peer":
            self.zc = self.peer.tensor(lay["zc"], (N, self.R, C_IN))
            self.zb = self.peer.tensor(lay["zb"], (self.P, self.R, self.R, C_IN))
            self.ws = self.peer.tensor(lay["ws"], (self.w.total,), torch.uint8)
            t_start, t_end, flags = peer_block_tables(self.peer.ptrs, self.rank, N, self.P)
            self.tab_start = torch.tensor(t_start, dtype=torch.int64, device=device)
            self.tab_end = torch.tensor(t_end, dtype=torch.int64, device=device)
            self.flag_tab = torch.tensor(flags, dtype=torch.int64, device=device)
            self.buf_tab = torch.tensor(self.peer.ptrs, dtype=torch.int64, device=device)
            self.epoch = 0
            self.send = self.zb
        else:
            self.ws = torch.empty(self.w.total, dtype=torch.uint8, device=device)
            self.send = torch.empty(self.P, self.R, self.R, C_IN, device=device)
            self.recv = torch.empty_like(self.send)
            self.recv2 = torch.empty_like(self.send)

    def _need_nccl(self) -> None:
        if self.exchange != "nccl":
            raise RuntimeError("this entry point uses the all-to-all exchange; the peer exchange runs pair_blocks")

    def close(self) -> None:
        """Release the shared buffers of the peer exchange (every rank, after the GPU work)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def barrier(self) -> None:
        """Cross-GPU barrier on the current stream (peer exchange)."""
        self.epoch += 1
        _lib.check(self.L.triattn_peer_barrier(self.flag_tab.data_ptr(), self.rank, self.P, self.epoch, self._st()))

    def share_bias(self) -> None:
        """Peer exchange: store this rank's tri-bias rows into every other rank's workspace (one
        launch over NVLink), then a barrier: the all-gather of the NCCL exchange."""
        b0, b1 = self.w.bias_rows(self.r0, self.r1)
        _lib.check(self.L.triattn_peer_broadcast(self.buf_tab.data_ptr(), self.rank, self.P, self.lay["ws"] + b0,
                                                 b1 - b0, self._st()))
        self.barrier()

    def _st(self):
        return _lib.stream_handle(self.device)

    def start(self, z_loc: torch.Tensor, mask: Optional[torch.Tensor], packed: torch.Tensor) -> None:
        """z_loc [R, N, 128] (rows r0..r1 of z) += TriAttStart(z) for those rows, in place."""
        self._need_nccl()
        L, N, R, r0, r1, dt, st = self.L, self.N, self.R, self.r0, self.r1, self.dt, self._st()
        ws, nb = self.ws.data_ptr(), self.ws.numel()
        mptr = None if mask is None else mask.data_ptr() + r0 * N * 4
        _lib.check(L.triattn_mask_prep_v(mptr, N * N, N, 1, 1, N, self.inf, r0, r1, dt, ws, nb, st))
        _lib.check(L.triattn_ln_proj_v(z_loc.data_ptr(), R * N * C_IN, N * C_IN, C_IN, packed.data_ptr(), 1, N, r0, r1,
                                       dt, ws, nb, st))
        gather_bias(self.ws, self.w, r0, r1, self.group)
        _lib.check(L.triattn_core(1, N, r0, r1, dt, ws, nb, st))
        zp = z_loc.data_ptr()
        _lib.check(L.triattn_out_proj_v(zp, R * N * C_IN, N * C_IN, C_IN, zp, R * N * C_IN, N * C_IN, C_IN,
                                        packed.data_ptr(), 1, N, r0, r1, dt, 1, ws, nb, st))

    def end(self, z_loc: torch.Tensor, mask: Optional[torch.Tensor], packed: torch.Tensor) -> None:
        """z_loc [R, N, 128] += TriAttEnd(z) for rows r0..r1, via the column block of z."""
        self._need_nccl()
        L, N, R, r0, r1, dt, st = self.L, self.N, self.R, self.r0, self.r1, self.dt, self._st()
        ws, nb = self.ws.data_ptr(), self.ws.numel()
        zt = rows_to_cols(z_loc, self.P, self.send, self.recv, self.group)  # [N, R, 128]
        # attention row a (global, in [r0, r1)) is column a of z: x_att[a][c] = zt[c][a - r0]
        mptr = None if mask is None else mask.data_ptr() + r0 * 4
        _lib.check(L.triattn_mask_prep_v(mptr, N * N, 1, N, 1, N, self.inf, r0, r1, dt, ws, nb, st))
        zp = zt.data_ptr()
        _lib.check(L.triattn_ln_proj_v(zp, N * R * C_IN, C_IN, R * C_IN, packed.data_ptr(), 1, N, r0, r1, dt, ws, nb,
                                       st))
        gather_bias(self.ws, self.w, r0, r1, self.group)
        _lib.check(L.triattn_core(1, N, r0, r1, dt, ws, nb, st))
        _lib.check(L.triattn_out_proj_v(zp, N * R * C_IN, C_IN, R * C_IN, zp, N * R * C_IN, C_IN, R * C_IN,
                                        packed.data_ptr(), 1, N, r0, r1, dt, 1, ws, nb, st))
        cols_to_rows(zt, self.P, self.recv2, z_loc, self.group)

    def start_blocks(self, z_blk: torch.Tensor, mask: Optional[torch.Tensor], packed: torch.Tensor) -> None:
        """z_blk [P, R, R, 128] (my rows of z, column blocks) += TriAttStart(z) for those rows, in place."""
        self._need_nccl()
        L, N, R, r0, r1, dt, st = self.L, self.N, self.R, self.r0, self.r1, self.dt, self._st()
        ws, nb = self.ws.data_ptr(), self.ws.numel()
        mptr = None if mask is None else mask.data_ptr() + r0 * N * 4
        _lib.check(L.triattn_mask_prep_v(mptr, N * N, N, 1, 1, N, self.inf, r0, r1, dt, ws, nb, st))
        zp = z_blk.data_ptr()
        s_row, s_col, cb, s_cb = R * C_IN, C_IN, R, R * R * C_IN
        _lib.check(L.triattn_ln_proj_vb(zp, N * N * C_IN, s_row, s_col, cb, s_cb, packed.data_ptr(), 1, N, r0, r1, dt,
                                        ws, nb, st))
        gather_bias(self.ws, self.w, r0, r1, self.group)
        _lib.check(L.triattn_core(1, N, r0, r1, dt, ws, nb, st))
        _lib.check(L.triattn_out_proj_vb(zp, N * N * C_IN, s_row, s_col, cb, s_cb, zp, N * N * C_IN, s_row, s_col, cb,
                                         s_cb, packed.data_ptr(), 1, N, r0, r1, dt, 1, ws, nb, st))

    def end_blocks(self, z_blk: torch.Tensor, mask: Optional[torch.Tensor], packed: torch.Tensor) -> None:
        """z_blk += TriAttEnd(z) for my rows: all-to-all to my column block, the layer on it in place,
        all-to-all straight back into z_blk."""
        self._need_nccl()
        L, N, R, r0, r1, dt, st = self.L, self.N, self.R, self.r0, self.r1, self.dt, self._st()
        ws, nb = self.ws.data_ptr(), self.ws.numel()
        zt = blocks_to_cols(z_blk, self.recv, self.group)  # [N, R, 128]
        mptr = None if mask is None else mask.data_ptr() + r0 * 4
        _lib.check(L.triattn_mask_prep_v(mptr, N * N, 1, N, 1, N, self.inf, r0, r1, dt, ws, nb, st))
        zp = zt.data_ptr()
        _lib.check(L.triattn_ln_proj_v(zp, N * R * C_IN, C_IN, R * C_IN, packed.data_ptr(), 1, N, r0, r1, dt, ws, nb,
                                       st))
        gather_bias(self.ws, self.w, r0, r1, self.group)
        _lib.check(L.triattn_core(1, N, r0, r1, dt, ws, nb, st))
        _lib.check(L.triattn_out_proj_v(zp, N * R * C_IN, C_IN, R * C_IN, zp, N * R * C_IN, C_IN, R * C_IN,
                                        packed.data_ptr(), 1, N, r0, r1, dt, 1, ws, nb, st))
        cols_to_blocks(zt, z_blk, self.group)

    def start_peer(self, mask: Optional[torch.Tensor], packed: torch.Tensor) -> None:
        """Starting node on zb (my rows, column blocks); the output z + y goes straight into the column
        buffers zc of the owning ranks, then a barrier."""
        L, N, R, r0, r1, dt, st = self.L, self.N, self.R, self.r0, self.r1, self.dt, self._st()
        ws, nb = self.ws.data_ptr(), self.ws.numel()
        mptr = None if mask is None else mask.data_ptr() + r0 * N * 4
        _lib.check(L.triattn_mask_prep_v(mptr, N * N, N, 1, 1, N, self.inf, r0, r1, dt, ws, nb, st))
        zp = self.zb.data_ptr()
        s_row, s_col, cb, s_cb = R * C_IN, C_IN, R, R * R * C_IN
        _lib.check(L.triattn_ln_proj_vb(zp, N * N * C_IN, s_row, s_col, cb, s_cb, packed.data_ptr(), 1, N, r0, r1, dt,
                                        ws, nb, st))
        self.share_bias()
        _lib.check(L.triattn_core(1, N, r0, r1, dt, ws, nb, st))
        _lib.check(L.triattn_out_proj_vt(zp, N * N * C_IN, s_row, s_col, cb, s_cb, self.zc.data_ptr(), N * R * C_IN,
                                         R * C_IN, C_IN, R, self.tab_start.data_ptr(), packed.data_ptr(), 1, N, r0,
                                         r1, dt, 1, ws, nb, st))
        self.barrier()

    def end_peer(self, mask: Optional[torch.Tensor], packed: torch.Tensor) -> None:
        """Ending node on zc (my columns); the output goes straight back into the row owners' zb,
        then a barrier."""
        L, N, R, r0, r1, dt, st = self.L, self.N, self.R, self.r0, self.r1, self.dt, self._st()
        ws, nb = self.ws.data_ptr(), self.ws.numel()
        mptr = None if mask is None else mask.data_ptr() + r0 * 4
        _lib.check(L.triattn_mask_prep_v(mptr, N * N, 1, N, 1, N, self.inf, r0, r1, dt, ws, nb, st))
        zp = self.zc.data_ptr()
        _lib.check(L.triattn_ln_proj_v(zp, N * R * C_IN, C_IN, R * C_IN, packed.data_ptr(), 1, N, r0, r1, dt, ws, nb,
                                       st))
        self.share_bias()
        _lib.check(L.triattn_core(1, N, r0, r1, dt, ws, nb, st))
        _lib.check(L.triattn_out_proj_vt(zp, N * R * C_IN, C_IN, R * C_IN, 0, 0, self.zb.data_ptr(), N * N * C_IN,
                                         C_IN, R * C_IN, R, self.tab_end.data_ptr(), packed.data_ptr(), 1, N, r0, r1,
                                         dt, 1, ws, nb, st))
        self.barrier()

    def check_status(self, when: str) -> None:
        """Raise TriAttnError on EVERY rank when the device status word of ANY rank holds an error (one
        small all-reduce MAX, so no rank goes on into the next exchange while another has stopped).  The
        word is cleared on read, so the next pair starts clean."""
        own = _lib.device_status(clear=True)
        v = torch.tensor([own], dtype=torch.int32, device=self.device)
        dist.all_reduce(v, op=dist.ReduceOp.MAX, group=self.group)
        worst = int(v.item())
        if worst != 0:
            raise _lib.TriAttnError(_lib.EDEVICE, f"device status {worst} {when} (this rank {self.rank} of {self.P}: "
                                                  f"{own}; 106 = a cross-GPU barrier ran out of time)")

    def pair_blocks(self, z_blk, mask, packed_start, packed_end) -> None:
        """One start+end pair on the block-layout residual stream.  nccl: two all-to-alls, no copies.
        peer: z_blk should be self.zb (the shared buffer; anything else is copied in and out).
        checked mode: an error recorded before the pair raises before any launch; one recorded during
        the pair raises after it (the blocks are then not to be used)."""
        if self.checked:
            self.check_status("before the pair")
        if self.exchange == "peer":
            own = z_blk.data_ptr() == self.zb.data_ptr()
            if not own:
                self.zb.copy_(z_blk)
            self.start_peer(mask, packed_start)
            self.end_peer(mask, packed_end)
            if self.checked:
                self.check_status("after the pair")
            if not own:
                z_blk.copy_(self.zb)
            return
        self.start_blocks(z_blk, mask, packed_start)
        self.end_blocks(z_blk, mask, packed_end)
        if self.checked:
            self.check_status("after the pair")

    def pair(self, z_loc, mask, packed_start, packed_end) -> None:
        """One start+end pair on a row-layout shard z_loc [R, N, 128] (converted to blocks and back)."""
        to_blocks(z_loc, self.P, self.send)
        self.pair_blocks(self.send, mask, packed_start, packed_end)
        from_blocks(self.send, z_loc)

    def nvlink_bytes_per_pair(self) -> int:
        """Bytes each rank sends over NVLink per pair: 2 tri-bias all-gathers (its own bias rows to each
        of the P - 1 peers) + 2 exchanges of fp32 z blocks (all-to-alls, or the same bytes as peer
        stores)."""
        b0, b1 = self.w.bias_rows(self.r0, self.r1)
        bias = (self.P - 1) * (b1 - b0)
        a2a = (self.P - 1) * self.R * self.R * C_IN * 4
        return 2 * bias + 2 * a2a


def _time_sharded_pair(cfg_id, args, dev, make_config_inputs, layer_flops, peaks):
    """Build a ShardedPair for configuration cfg_id, time args.steps pairs (max over ranks) and the attention
    core alone; returns (record dict, sp, packs, mask, z_loc, z_h, pm_h, stream).  The caller closes sp."""
    from .triangle_attention import TriangleAttention, load_params

    z_h, pm_h, ps, pe = make_config_inputs(cfg_id)
    N = z_h.shape[1]
    prec = args.precision or {0: "fp32", 1: "fp16"}.get(cfg_id, "bf16")
    # unchecked in the timed loop (no host sync per step); the status is read on every rank at the end
    sp = ShardedPair(N, prec, dev, exchange=getattr(args, "exchange", "peer"), checked=False)
    exchange = sp.exchange  # "nccl" if the peer mappings were refused on some rank
    packs = []
    for starting, p in ((True, ps), (False, pe)):
        m = TriangleAttention(starting=starting, precision=prec).to(dev)
        load_params(m, {k: (v.to(dev) if v is not None else None) for k, v in p.items()})
        packs.append(m.packed_weights(sp.dt))
    mask = pm_h[0].contiguous().to(dev)
    z_loc = z_h[0, sp.r0:sp.r1].contiguous().to(dev)
    # the residual stream stays in block layout across steps (the layout the exchange uses)
    z_blk = to_blocks(z_loc, sp.P, sp.zb if exchange == "peer" else torch.empty(sp.P, sp.R, sp.R, C_IN, device=dev))

    def step():  # in place: every step is the same work on the updated shard
        sp.pair_blocks(z_blk, mask, packs[0], packs[1])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(dev)
    dist.barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = torch.tensor([ev0.elapsed_time(ev1) / args.steps], device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    step_ms = float(ms)
    fl = layer_flops(N)
    pair_flops = 2 * fl["total"]

    # dominant kernel: the attention core on this rank's rows (end-layer workspace), timed alone;
    # max over ranks
    st = _lib.stream_handle(dev)
    L = _lib.lib()
    for _ in range(2):
        _lib.check(L.triattn_core(1, N, sp.r0, sp.r1, sp.dt, sp.ws.data_ptr(), sp.ws.numel(), st))
    ev0.record(stream)
    for _ in range(5):
        _lib.check(L.triattn_core(1, N, sp.r0, sp.r1, sp.dt, sp.ws.data_ptr(), sp.ws.numel(), st))
    ev1.record(stream)
    torch.cuda.synchronize()
    core = torch.tensor([ev0.elapsed_time(ev1) / 5], device=dev)
    dist.all_reduce(core, op=dist.ReduceOp.MAX)
    core_ms = float(core)
    pk, pk_kind = peaks()
    tensor_peak = pk.get("bf16_tflops", 1590.0)
    achieved = fl["core"] * sp.R / N / (core_ms * 1e-3) / 1e12
    traffic = None
    tf = Path(__file__).resolve().parents[1] / "profiles" / "core_traffic.json"
    if tf.exists():
        try:
            full = json.loads(tf.read_text()).get(str(N))
            # one core launch's DRAM bytes at this N (ncu, all N rows), scaled to this rank's R rows: the
            # core reads each row's q, k, v images and writes its output once, so traffic grows with R
            traffic = None if full is None else full * sp.R / N
        except ValueError:
            traffic = None
    rec = {"N": N, "precision": prec, "ms_per_step": step_ms, "ms_per_layer": step_ms / 2,
           "tflops": pair_flops / (step_ms * 1e-3) / 1e12, "rows_per_rank": sp.R,
           "nvlink_bytes_per_rank_per_step": sp.nvlink_bytes_per_pair(),
           "exchange": {"peer": "peer stores from the output projection + cross-GPU barrier (CUDA IPC)",
                        "nccl": "NCCL all_to_all_single"}[exchange],
           "roofline": {"bound": "tensor", "kernel": "core_tc (flash attention core, this rank's rows)",
                        "achieved": achieved, "peak": tensor_peak, "unit": "TFLOP/s",
                        "frac": achieved / tensor_peak, "peak_kind": f"{pk_kind} bf16 burst, per GPU",
                        "traffic": traffic,
                        "traffic_note": "ncu DRAM bytes of one full-N core launch (profiles/core_traffic.json) x R/N",
                        "core_ms": core_ms,
                        "algorithmic": f"F_core * R / N = {fl['core'] * sp.R / N:.4g} FLOP per launch"},
           "gpu_launches": args.steps * 2 * (7 if exchange == "peer" else 4)}
    return rec, sp, packs, mask, z_loc, z_h, pm_h, stream


def bench_sharded(args, make_config_inputs, layer_flops, workload_config, metric_name, ClockSampler,
                  physical_gpu_index, peaks):
    """bench.py --gpus P under torchrun: one start+end pair on the row-sharded pair tensor per step; the
    headline configuration, then (for config 2) config 4 (N=2048) at the same P as a nested record."""
    from datetime import timedelta

    ws_n = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    sp = None
    try:
        with ClockSampler(physical_gpu_index(local)) as clk:
            rec, sp, packs, mask, z_loc, z_h, pm_h, stream = _time_sharded_pair(
                args.config, args, dev, make_config_inputs, layer_flops, peaks)
        N, prec, step_ms = rec["N"], rec["precision"], rec["ms_per_step"]
        fl = layer_flops(N)
        pair_flops = 2 * fl["total"]
        value = pair_flops / (step_ms * 1e-3) / 1e12
        # e2e: host shard + mask copied in, shard copied out, every step; consecutive steps are
        # pipelined over two device slots (input copy / pair / output copy on three streams)
        zh = z_h[0, sp.r0:sp.r1].contiguous().pin_memory()
        mh = pm_h[0].contiguous().pin_memory()
        ohs = [torch.empty_like(zh).pin_memory() for _ in range(2)]
        zls = [z_loc, torch.empty_like(z_loc)]
        mks = [mask, torch.empty_like(mask)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_comp = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        for e_ in ev_comp + ev_out:
            e_.record(stream)

        def e2e_step(k):
            s_ = k % 2
            with torch.cuda.stream(s_in):
                s_in.wait_event(ev_comp[s_])
                zls[s_].copy_(zh, non_blocking=True)
                mks[s_].copy_(mh, non_blocking=True)
                ev_in[s_].record(s_in)
            stream.wait_event(ev_in[s_])
            stream.wait_event(ev_out[s_])
            sp.pair(zls[s_], mks[s_], packs[0], packs[1])
            ev_comp[s_].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_comp[s_])
                ohs[s_].copy_(zls[s_], non_blocking=True)
                ev_out[s_].record(s_out)

        for k in range(2):
            e2e_step(k)
        torch.cuda.synchronize()
        dist.barrier()
        # window: first input copy to last output copy (one pipeline fill included), over enough steps to
        # keep the fill's share small; the steady-state period between output copies is reported beside it
        n_e2e = min(max(10, 2 * args.steps), 40)
        t0, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        done = [torch.cuda.Event(enable_timing=True) for _ in range(n_e2e)]
        t0.record(s_in)
        for k in range(n_e2e):
            e2e_step(k)
            done[k].record(s_out)
        t1e.record(s_out)
        torch.cuda.synchronize()
        e2e = torch.tensor([t0.elapsed_time(t1e) / n_e2e, done[2].elapsed_time(done[-1]) / (n_e2e - 3)], device=dev)
        dist.all_reduce(e2e, op=dist.ReduceOp.MAX)
        oh = ohs[0]
        status = torch.tensor([_lib.device_status()], device=dev)
        dist.all_reduce(status, op=dist.ReduceOp.MAX)
        nested = None
        if args.config == 2:
            # the north star's scaling target is quoted at N=2048 (config 4): the same pair at the same P
            sp.close()
            sp = None
            torch.cuda.empty_cache()
            nested, sp, *_ = _time_sharded_pair(4, args, dev, make_config_inputs, layer_flops, peaks)
            st4 = torch.tensor([_lib.device_status()], device=dev)
            dist.all_reduce(st4, op=dist.ReduceOp.MAX)
            nested["device_status"] = int(st4)
            nested["metric"] = metric_name(4)
            nested["config"] = workload_config(4, ws_n)
        if rank == 0:
            line = {
                "metric": metric_name(args.config), "value": value, "unit": "TFLOP/s", "n_gpus": ws_n,
                "gpu": torch.cuda.get_device_name(dev), "host_cores": os.cpu_count(),
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms, "ms_per_layer": step_ms / 2,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": prec,
                "data": "synthetic: z~N(0,1)*scale, seeded trailing-padding pair mask, seeded N(0,1/128) weights",
                "config": workload_config(args.config, ws_n),
                "nvlink_bytes_per_rank_per_step": rec["nvlink_bytes_per_rank_per_step"],
                "exchange": rec["exchange"],
                "roofline": rec["roofline"],
                "cpu_baseline": {"note": "timed on rank 0 of the 1-GPU run only (the same host and workload)"},
                "e2e": {"value": pair_flops / (float(e2e[0]) * 1e-3) / 1e12, "unit": "TFLOP/s",
                        "ms_per_step": float(e2e[0]), "h2d_bytes_per_step": (zh.numel() + mh.numel()) * 4 * ws_n,
                        "d2h_bytes_per_step": oh.numel() * 4 * ws_n,
                        "pipelined": "input copy, pair and output copy of consecutive steps overlap (2 device slots)",
                        "steps": n_e2e, "ms_per_step_steady": float(e2e[1]),
                        "window": "first input copy to last output copy (one pipeline fill included), max over "
                                  "ranks; ms_per_step_steady = period between consecutive output copies after the fill"},
                "gpu_launches": rec["gpu_launches"],
                "device_status": int(status),
                "clocks": clk.summary(),
            }
            if nested is not None:
                line["config4_same_gpus"] = nested
            print(json.dumps(line), flush=True)
    finally:
        if sp is not None:
            sp.close()
        dist.barrier()
        dist.destroy_process_group()
