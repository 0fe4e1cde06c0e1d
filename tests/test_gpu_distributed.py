"""GPU: the row-sharded start+end pair equals the single-GPU pair bit for bit (the per-row arithmetic
is identical; only the data movement differs), with either exchange: NCCL all-to-alls, or peer stores
from the output projection plus the cross-GPU barrier.  2 ranks need 2 GPUs (skipped otherwise); the
peer path with one rank (its own buffer as the only peer) runs on one GPU.  The barrier's bounded wait
is made to run out on purpose with a flag slot that nothing sets: it must record status 106 and leave
the context usable."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, P, port, N, precision, errq, exchange="nccl", steps=1):
    try:
        import torch.distributed as dist
        from datetime import timedelta

        from boltz_mlx_b200 import TriangleAttention, _lib, load_params
        from boltz_mlx_b200.distributed import ShardedPair
        from oracle.triattn_ref import make_params
        from tests._util import rand_mask

        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=P, timeout=timedelta(seconds=60), device_id=dev)
        g = torch.Generator().manual_seed(21)
        z = torch.randn(1, N, N, 128, generator=g)
        m = rand_mask(g, 1, N)
        mods = []
        for starting, seed in ((True, 1), (False, 2)):
            mod = TriangleAttention(starting=starting, precision=precision).to(dev)
            load_params(mod, {k: (v.to(dev) if v is not None else None)
                              for k, v in make_params(seed, gate_bias=1.0).items()})
            mods.append(mod)
        zc, mc = z.to(dev), m.to(dev)
        full = zc
        for _ in range(steps):
            full = mods[1].forward_residual(mods[0].forward_residual(full, mc), mc)
        sp = ShardedPair(N, precision, dev, exchange=exchange)
        try:
            dt = _lib.dtype_code(precision)
            z_loc = zc[0, sp.r0:sp.r1].contiguous()
            for _ in range(steps):
                sp.pair(z_loc, mc[0].contiguous(), mods[0].packed_weights(dt), mods[1].packed_weights(dt))
            torch.cuda.synchronize()
            assert _lib.device_status() == 0
            assert torch.equal(z_loc, full[0, sp.r0:sp.r1]), float((z_loc - full[0, sp.r0:sp.r1]).abs().max())
        finally:
            sp.close()
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {e!r}")
        raise


def _run(P, N, precision, exchange, steps):
    ctx = torch.multiprocessing.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, P, port, N, precision, errq, exchange, steps)) for r in range(P)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "peer"])
@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_sharded_pair_equals_single_gpu(precision, exchange):
    _run(2, 256, precision, exchange, steps=2 if exchange == "peer" else 1)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_peer_exchange_one_rank_equals_single_gpu(precision):
    _run(1, 256, precision, "peer", steps=2)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_peer_barrier_times_out_without_a_peer():
    """Two flag blocks on this GPU; rank 0 of a 2-rank barrier signals both, but nothing ever signals
    its slot for rank 1, so lane 1's wait runs out: status 106, then the context still works."""
    from boltz_mlx_b200 import _lib

    L = _lib.lib()
    dev = torch.device("cuda", 0)
    flags = torch.zeros(2, 64, dtype=torch.int32, device=dev)  # two blocks of slots, 256 B apart
    tab = torch.tensor([flags[0].data_ptr(), flags[1].data_ptr()], dtype=torch.int64, device=dev)
    assert _lib.device_status() == 0
    _lib.check(L.triattn_peer_barrier(tab.data_ptr(), 0, 2, 1, _lib.stream_handle(dev)))
    assert _lib.device_status() == 106
    assert int(flags[0, 0]) == 1 and int(flags[1, 0]) == 1  # both signals went out
    # a satisfied barrier afterwards: a 1-rank group over its own block
    _lib.check(L.triattn_peer_barrier(tab.data_ptr(), 0, 1, 2, _lib.stream_handle(dev)))
    assert _lib.device_status() == 0
    x = torch.ones(1024, device=dev)
    assert float(x.sum()) == 1024.0


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4, reason="needs 4 GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_sharded_pair_four_ranks(exchange):
    _run(4, 512, "bf16", exchange, steps=2)
