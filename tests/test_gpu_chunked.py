"""GPU: the row-chunked layer (large-N memory path; the reference's chunking, attention.py:55-68).

triattn_forward_chunked and the module's automatic chunking give the whole-layer result bit for bit
(per-row arithmetic is identical; only the row ranges of the calls differ), on ragged chunk sizes, both
nodes, in place and out of place.  At N = 2304 the pair tensor is 2.7 GB, so element offsets into z
and out pass 2^31 bytes (the 64-bit indexing the reference's report flags at 2^31, docs/report.md:164);
the last attention row (the largest offsets) is checked against the oracle."""

import pytest
import torch

from boltz_mlx_b200 import _lib
from oracle.triattn_ref import make_params, tri_attention_ref
from tests._util import assert_parity, module, rand_mask

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0


@pytest.mark.parametrize("precision,chunk", [("fp32", 100), ("bf16", 128), ("fp16", 256)])
def test_chunked_entry_equals_whole_layer(precision, chunk):
    N = 300
    g = torch.Generator().manual_seed(23)
    z = torch.randn(1, N, N, 128, generator=g).cuda()
    m = rand_mask(g, 1, N).cuda()
    dt = _lib.dtype_code(precision)
    L, st = _lib.lib(), _lib.stream_handle(z.device)
    for starting in (True, False):
        mod = module(make_params(5, gate_bias=1.0), starting, precision)
        packed = mod.packed_weights(dt)
        whole = mod.forward_residual(z, m)
        ws = torch.empty(_lib.workspace_bytes(1, N, chunk, dt), dtype=torch.uint8, device="cuda")
        out = torch.empty_like(z)
        _lib.check(L.triattn_forward_chunked(z.data_ptr(), m.data_ptr(), packed.data_ptr(), 1, N, int(starting), 1e9,
                                             dt, 1, out.data_ptr(), chunk, ws.data_ptr(), ws.numel(), st))
        assert torch.equal(out, whole)
        zi = z.clone()  # in place: out aliases z
        _lib.check(L.triattn_forward_chunked(zi.data_ptr(), m.data_ptr(), packed.data_ptr(), 1, N, int(starting), 1e9,
                                             dt, 1, zi.data_ptr(), chunk, ws.data_ptr(), ws.numel(), st))
        assert torch.equal(zi, whole)
        # a workspace for fewer rows than the chunk is refused
        small = _lib.workspace_bytes(1, N, chunk, dt) - 256
        assert L.triattn_forward_chunked(z.data_ptr(), m.data_ptr(), packed.data_ptr(), 1, N, int(starting), 1e9, dt,
                                         1, out.data_ptr(), chunk, ws.data_ptr(), small, st) == _lib.ENOSPACE


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_module_chunk_size_equals_whole(precision):
    N = 260
    g = torch.Generator().manual_seed(29)
    z = torch.randn(1, N, N, 128, generator=g).cuda()
    m = rand_mask(g, 1, N).cuda()
    for starting in (True, False):
        mod = module(make_params(6, gate_bias=1.0), starting, precision)
        assert torch.equal(mod(z, m, chunk_size=128), mod(z, m))
        mod.max_workspace_bytes = _lib.workspace_bytes(1, N, 128, _lib.dtype_code(precision))  # forces chunks
        assert mod.chunk_rows(1, N, _lib.dtype_code(precision)) == 128
        assert torch.equal(mod(z, m), mod(z, m, chunk_size=N))


def test_large_n_chunked_bf16():
    N = 2304
    g = torch.Generator().manual_seed(31)
    z = (0.5 * torch.randn(1, N, N, 128, generator=g))
    m = torch.ones(1, N, N)
    m[:, :, N - 100:] = 0.0  # padded key columns
    m[:, N - 100:, :] = 0.0  # padded rows (the last rows attend uniformly)
    p = make_params(7, gate_bias=1.0)
    zc, mc = z.cuda(), m.cuda()
    for starting in (True, False):
        mod = module(p, starting, "bf16")
        mod.max_workspace_bytes = 2 << 30
        rows = mod.chunk_rows(1, N, _lib.BF16)
        assert rows < N and rows % 128 == 0
        y = mod(zc, mc)
        assert torch.equal(y, mod(zc, mc, chunk_size=N))
        ya = y if starting else y.transpose(1, 2)
        for r in (N - 101, N - 1):  # last valid row and the last row: the largest offsets into z / out
            ref = tri_attention_ref(z, m, p, starting=starting, rows=(r, r + 1))
            assert_parity(ya[:, r:r + 1].cpu(), ref, "bf16", f"N={N} start={starting} row {r}")
        del y, ya
        torch.cuda.empty_cache()
