"""CPU, multi-process (gloo): the row-sharded layer's exchange steps -- the tri-bias all-gather and
the all-to-all row <-> column re-sharding -- against single-process references, world sizes 2 and 4.
The same functions drive the NCCL path on the GPUs."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from boltz_mlx_b200.distributed import (all_ranks_ok, blocks_to_cols, cols_to_blocks, cols_to_rows,
                                        exchange_intact, from_blocks, gather_bias, rows_to_cols, shard_rows,
                                        to_blocks)
from boltz_mlx_b200.layout import Workspace


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, P, port, N, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=P)
        C = 8
        g = torch.Generator().manual_seed(0)
        z = torch.randn(N, N, C, generator=g)  # every rank builds the same full tensor
        r0, r1 = shard_rows(N, P, rank)
        R = r1 - r0
        send = torch.empty(P, R, R, C)
        recv = torch.empty_like(send)
        recv2 = torch.empty_like(send)
        z_loc = z[r0:r1].clone()
        zt = rows_to_cols(z_loc, P, send, recv)
        assert torch.equal(zt, z[:, r0:r1]), "rows_to_cols"
        zt.mul_(2.0).add_(float(rank))  # a column-block update
        out = torch.empty_like(z_loc)
        cols_to_rows(zt, P, recv2, out)
        ref = z * 2.0
        for q in range(P):
            ref[:, q * R:(q + 1) * R] += float(q)
        assert torch.equal(out, ref[r0:r1]), "cols_to_rows"
        # block layout of the residual stream: z_blk[p, i, a] = z[r0 + i, p*R + a]; the all-to-all
        # sends block p to rank p as-is and the column block comes back into the same layout
        z_blk = to_blocks(z_loc, P, torch.empty(P, R, R, C))
        for q in range(P):
            assert torch.equal(z_blk[q], z[r0:r1, q * R:(q + 1) * R]), "to_blocks"
        assert torch.equal(from_blocks(z_blk, torch.empty_like(z_loc)), z_loc), "from_blocks"
        zt2 = blocks_to_cols(z_blk, torch.empty(P, R, R, C))
        assert torch.equal(zt2, z[:, r0:r1]), "blocks_to_cols"
        zt2.mul_(2.0).add_(float(rank))
        cols_to_blocks(zt2, z_blk)
        assert torch.equal(from_blocks(z_blk, torch.empty_like(z_loc)), ref[r0:r1]), "cols_to_blocks"
        # tri-bias all-gather over the workspace layout
        for dtype in (0, 2):
            if dtype != 0 and R % 128:
                continue  # 16-bit tri-bias rows move in 128-row blocks
            w = Workspace.make(1, N, R, dtype)
            ws = torch.zeros(w.total, dtype=torch.uint8)
            l0, l1 = w.bias_rows(r0, r1)
            ws[l0:l1] = (rank + 1) * torch.ones(l1 - l0, dtype=torch.uint8)
            ws[l1:] = 77  # per-row regions must not be touched
            gather_bias(ws, w, r0, r1)
            for q in range(P):
                a, b = w.bias_rows(q * R, (q + 1) * R)
                assert torch.all(ws[a:b] == q + 1), "gather_bias"
            b0, b1 = w.bias_rows(0, N)
            assert torch.all(ws[b1:] == 77)
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # report to the parent
        errq.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.parametrize("P,N", [(2, 8), (4, 12), (2, 256)])
def test_exchange_steps(P, N):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, P, port, N, errq)) for r in range(P)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_shard_rows_requires_divisibility():
    assert shard_rows(1024, 8, 3) == (384, 512)
    with pytest.raises(NotImplementedError):
        shard_rows(1000, 3, 0)


def _agree_worker(rank, P, port, bad, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=P)
        # every rank learns whether all ranks succeeded (the peer exchange's set-up vote)
        assert all_ranks_ok(True) is True
        assert all_ranks_ok(rank != bad) is (bad < 0)
        assert all_ranks_ok(False) is False
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.parametrize("P,bad", [(2, -1), (2, 1), (4, 2)])
def test_all_ranks_ok_is_a_collective_vote(P, bad):
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_agree_worker, args=(r, P, port, bad, errq)) for r in range(P)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def _validation_worker(port, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=0, world_size=1)
        from boltz_mlx_b200 import _lib
        from boltz_mlx_b200.distributed import ShardedPair

        try:
            ShardedPair(256, "bf16", torch.device("cpu"), exchange="allreduce")
            raise AssertionError("unknown exchange accepted")
        except ValueError:
            pass
        try:  # 16-bit tri-bias rows move in 128-row blocks: rows per rank must be a multiple of 128
            ShardedPair(200, "bf16", torch.device("cpu"))
            raise AssertionError("ragged 16-bit shard accepted")
        except _lib.TriAttnUnsupported:
            pass
        sp = ShardedPair(200, "fp32", torch.device("cpu"))  # fp32 shards take any row count
        assert (sp.r0, sp.r1, sp.exchange) == (0, 200, "nccl")
        sp.close()  # no peer buffers: a no-op
        dist.destroy_process_group()
    except Exception as e:
        errq.put(repr(e))
        raise


def test_sharded_pair_validates_its_arguments():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    p = ctx.Process(target=_validation_worker, args=(_free_port(), errq))
    p.start()
    p.join(timeout=120)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert p.exitcode == 0


def _fault_worker(rank, P, port, mode, errq):
    """mode 'corrupt': rank 1 damages one received block; every rank must see the exchange fail.
    mode 'absent': rank 1 leaves before the exchange; the others must get an error within the
    process-group timeout (no hang)."""
    from datetime import timedelta

    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=P, timeout=timedelta(seconds=5))
        R, C = 4, 8
        z_blk = torch.randn(P, R, R, C, generator=torch.Generator().manual_seed(rank))
        if mode == "absent" and rank == 1:
            return  # leaves without joining the exchange (the host-side stand-in for a dead rank)
        recv = torch.empty_like(z_blk)
        try:
            blocks_to_cols(z_blk, recv)
        except RuntimeError:
            assert mode == "absent", "the exchange failed without a fault"
            errq.put(f"ok rank {rank}: detected")
            return
        assert mode != "absent", "the exchange completed without the absent rank"
        assert exchange_intact(z_blk, recv), "intact exchange reported as damaged"
        # non-finite data sent intact is intact: every rank sends NaN / inf in one block
        z_nf = z_blk.clone()
        z_nf[0, 0, 0, 0] = float("nan")
        z_nf[-1, 0, 0, 1] = float("inf")
        recv_nf = torch.empty_like(z_nf)
        blocks_to_cols(z_nf, recv_nf)
        assert exchange_intact(z_nf, recv_nf), "non-finite but intact blocks reported as damaged"
        if rank == 1:
            recv[0, 0, 0, 0] += 1.0  # a corrupted shard
        assert exchange_intact(z_blk, recv) is False, "damaged block not detected"
        errq.put(f"ok rank {rank}: detected")
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.parametrize("mode", ["corrupt", "absent"])
def test_exchange_faults_are_detected_on_the_host(mode):
    P = 3
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_fault_worker, args=(r, P, port, mode, errq)) for r in range(P)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    msgs = []
    while not errq.empty():
        msgs.append(errq.get())
    bad = [m for m in msgs if not m.startswith("ok")]
    assert not bad, bad
    expect = P if mode == "corrupt" else P - 1
    assert sum(m.startswith("ok") for m in msgs) == expect, msgs


def _checked_pair_worker(rank, world, port, errq):
    """ShardedPair in checked mode on gloo ranks, with the library's status read faked on the host:
    a stale error on one rank makes EVERY rank raise before launching anything, and an error recorded
    during a pair makes every rank raise after it instead of returning the blocks."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from boltz_mlx_b200 import _lib
        from boltz_mlx_b200 import distributed as tdist

        sp = tdist.ShardedPair(256, "bf16", torch.device("cpu"))
        assert sp.checked
        launched = []
        sp.start_blocks = lambda *a: launched.append("start")
        sp.end_blocks = lambda *a: launched.append("end")
        z_blk = torch.zeros(world, sp.R, sp.R, 4)
        # 1) stale error on rank 1 only (e.g. an earlier barrier timed out there)
        reads = iter([106 if rank == 1 else 0])
        _lib.device_status = lambda clear=True: next(reads, 0)
        try:
            sp.pair_blocks(z_blk, None, None, None)
            raise AssertionError("stale status not reported")
        except _lib.TriAttnError as e:
            assert "106" in str(e), str(e)
        assert launched == [], launched
        # 2) clean before, an error recorded during the pair on rank 0
        reads = iter([0, 102 if rank == 0 else 0])
        _lib.device_status = lambda clear=True: next(reads, 0)
        try:
            sp.pair_blocks(z_blk, None, None, None)
            raise AssertionError("in-pair error not reported")
        except _lib.TriAttnError as e:
            assert "102" in str(e), str(e)
        assert launched == ["start", "end"], launched
        # 3) clean: the pair returns
        _lib.device_status = lambda clear=True: 0
        sp.pair_blocks(z_blk, None, None, None)
        assert launched == ["start", "end", "start", "end"]
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {e!r}")
        raise


def test_checked_pair_reports_device_errors_on_every_rank():
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_checked_pair_worker, args=(r, 2, port, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
