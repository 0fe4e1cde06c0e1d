"""GPU: the TriangleAttention module (through libtriattn.so) against the CPU oracle and the golden
fixtures, in fp32 (max_rel <= 1e-5) and 16-bit (max_abs <= 2e-2, mean_abs <= 5e-3) modes, on the
reference tests' shapes: tiny / ragged N, B = 2, fully masked rows, masked key columns, both nodes."""

import numpy as np
import pytest
import torch

from boltz_mlx_b200 import _lib
from oracle.triattn_ref import make_params, tri_attention_ref
from tests._util import assert_parity, module, rand_mask
from tests.test_oracle import golden_case, golden_cases

pytestmark = pytest.mark.gpu
PRECISIONS = ["fp32", "bf16", "fp16"]


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("starting", [True, False])
def test_golden_fixtures(precision, starting):
    d, names = golden_cases()
    for name in names:
        z, m, p = golden_case(d, name)
        mod = module(p, starting, precision)
        out = mod(z.cuda(), None if m is None else m.cuda())
        assert_parity(out, d[f"{name}_y_{'start' if starting else 'end'}"], precision, name)


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("N", [1, 2, 9, 17, 33, 37, 117, 128, 129, 200])
@pytest.mark.parametrize("starting", [True, False])
def test_module_vs_oracle(precision, N, starting):
    g = torch.Generator().manual_seed(1000 + N)
    B = 2 if N <= 33 else 1
    z = torch.randn(B, N, N, 128, generator=g)
    m = rand_mask(g, B, N, "rows_cols")
    p = make_params(N, gate_bias=1.0 if N % 2 else None, ln_identity=N % 3 == 0)
    ref = tri_attention_ref(z, m, p, starting=starting, dtype=torch.float64)
    out = module(p, starting, precision)(z.cuda(), m.cuda())
    assert_parity(out, ref, precision, f"N={N}")


@pytest.mark.parametrize("precision", PRECISIONS)
def test_no_mask_equals_all_ones(precision):
    N = 70
    g = torch.Generator().manual_seed(5)
    z = torch.randn(1, N, N, 128, generator=g).cuda()
    mod = module(make_params(5), True, precision)
    a = mod(z, None)
    b = mod(z, torch.ones(1, N, N, device="cuda"))
    assert torch.equal(a, b)


@pytest.mark.parametrize("precision", PRECISIONS)
def test_residual_and_inplace(precision):
    N = 96
    g = torch.Generator().manual_seed(6)
    z = torch.randn(1, N, N, 128, generator=g).cuda()
    m = rand_mask(g, 1, N).cuda()
    for starting in (True, False):
        mod = module(make_params(6, gate_bias=1.0), starting, precision)
        y = mod(z, m)
        zr = mod.forward_residual(z, m)
        torch.testing.assert_close(zr, z + y, rtol=0, atol=1e-6)
        zi = z.clone()
        out = mod.forward_residual(zi, m, inplace=True)
        assert out.data_ptr() == zi.data_ptr()
        torch.testing.assert_close(zi, z + y, rtol=0, atol=1e-6)


@pytest.mark.parametrize("precision", PRECISIONS)
def test_ending_node_equals_starting_on_transpose(precision):
    """Size-independent property: end(z) == start(z^T)^T, bit for bit (same arithmetic per row)."""
    N = 160
    g = torch.Generator().manual_seed(8)
    z = torch.randn(1, N, N, 128, generator=g).cuda()
    m = rand_mask(g, 1, N).cuda()
    p = make_params(8, gate_bias=1.0)
    ye = module(p, False, precision)(z, m)
    ys = module(p, True, precision)(z.transpose(1, 2).contiguous(), m.transpose(1, 2).contiguous())
    assert torch.equal(ye, ys.transpose(1, 2))


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_row_chunked_stages_equal_full(precision):
    """The reference's row chunking (attention.py:55-68, tests/test_chunking.py): rows processed in
    chunks with the tri bias of ALL rows gives the full-layer result."""
    from boltz_mlx_b200 import layout

    N, chunk = 150, 64
    g = torch.Generator().manual_seed(11)
    z = torch.randn(1, N, N, 128, generator=g).cuda()
    m = rand_mask(g, 1, N).cuda()
    for starting in (True, False):
        mod = module(make_params(11, gate_bias=1.0), starting, precision)
        full = mod(z, m)
        dt = _lib.dtype_code(precision)
        packed = mod.packed_weights(dt)
        L, st = _lib.lib(), _lib.stream_handle(z.device)
        out = torch.empty_like(z)
        bounds = [(r, min(r + chunk, N)) for r in range(0, N, chunk)]
        R = chunk
        w = layout.Workspace.make(1, N, R, dt)
        ws = torch.empty(w.total, dtype=torch.uint8, device="cuda")
        for r0, r1 in bounds:  # pass 1: tri-bias rows of every chunk
            _lib.check(L.triattn_ln_proj(z.data_ptr(), packed.data_ptr(), 1, N, int(starting), r0, r1, dt,
                                         ws.data_ptr(), ws.numel(), st))
        for r0, r1 in bounds:  # pass 2: chunk by chunk
            _lib.check(L.triattn_mask_prep(m.data_ptr(), 1, N, int(starting), 1e9, r0, r1, dt, ws.data_ptr(),
                                           ws.numel(), st))
            _lib.check(L.triattn_ln_proj(z.data_ptr(), packed.data_ptr(), 1, N, int(starting), r0, r1, dt,
                                         ws.data_ptr(), ws.numel(), st))
            _lib.check(L.triattn_core(1, N, r0, r1, dt, ws.data_ptr(), ws.numel(), st))
            _lib.check(L.triattn_out_proj(z.data_ptr(), packed.data_ptr(), 1, N, int(starting), r0, r1, dt, 0,
                                          out.data_ptr(), ws.data_ptr(), ws.numel(), st))
        torch.cuda.synchronize()
        assert torch.equal(out, full)
