"""GPU, 2 ranks (NCCL): the row-sharded start+end pair equals the single-GPU pair bit for bit (the
per-row arithmetic is identical; only the data movement differs).  Skipped with fewer than 2 GPUs."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, P, port, N, precision, errq):
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
        full = mods[1].forward_residual(mods[0].forward_residual(zc, mc), mc)
        sp = ShardedPair(N, precision, dev)
        dt = _lib.dtype_code(precision)
        z_loc = zc[0, sp.r0:sp.r1].contiguous()
        sp.pair(z_loc, mc[0].contiguous(), mods[0].packed_weights(dt), mods[1].packed_weights(dt))
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        assert torch.equal(z_loc, full[0, sp.r0:sp.r1]), float((z_loc - full[0, sp.r0:sp.r1]).abs().max())
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        errq.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("precision", ["bf16", "fp32"])
def test_sharded_pair_equals_single_gpu(precision):
    P, N = 2, 256
    ctx = torch.multiprocessing.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, P, port, N, precision, errq)) for r in range(P)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
