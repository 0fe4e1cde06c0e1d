"""triattn_forward_noalloc: the triangle-attention layer for callers that cannot allocate device memory
while they run (their scratch comes from a fixed array inside libtriattn.so instead of a workspace they
pass in).  Its output must equal triattn_forward's bit for bit on the same inputs, call after call, and calls too
large for the fixed array must be refused before any work is launched.

This file is collected last on purpose (pytest orders test files by name), so a run that stops at the
first failure has already run every other test."""

import ctypes

import pytest
import torch

from boltz_mlx_b200 import _lib, layout
from oracle.triattn_ref import make_params
from tests._util import module, rand_mask


def _noalloc():
    L = _lib.lib()
    f = L.triattn_forward_noalloc
    vp, i, fl = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    f.argtypes = [vp, vp, vp, i, i, i, fl, i, i, vp, vp]
    f.restype = ctypes.c_int
    return f


@pytest.mark.gpu
@pytest.mark.parametrize("precision", ["bf16", "fp16", "fp32"])
def test_noalloc_matches_forward_on_consecutive_calls(precision):
    f = _noalloc()
    dt = _lib.dtype_code(precision)
    st = _lib.stream_handle(torch.device("cuda", 0))
    # two calls in a row with different shapes, orientations and masks: the second call starts from
    # whatever the first one left in the shared scratch array
    cases = [(True, 96, True, 1), (False, 128, False, 2), (True, 37, True, 3)]
    for starting, N, masked, seed in cases:
        g = torch.Generator().manual_seed(seed)
        z = torch.randn(1, N, N, 128, generator=g).cuda()
        m = rand_mask(g, 1, N).cuda() if masked else None
        mod = module(make_params(seed, gate_bias=1.0), starting, precision)
        packed = mod.packed_weights(dt)
        ref = torch.empty_like(z)
        ws = torch.empty(layout.workspace_bytes(1, N, N, dt), dtype=torch.uint8, device="cuda")
        _lib.check(_lib.lib().triattn_forward(z.data_ptr(), _lib.ptr(m), packed.data_ptr(), 1, N, int(starting), 1e9,
                                              dt, 1, ref.data_ptr(), ws.data_ptr(), ws.numel(), st))
        out = torch.full_like(z, float("nan"))
        _lib.check(f(z.data_ptr(), _lib.ptr(m), packed.data_ptr(), 1, N, int(starting), 1e9, dt, 1, out.data_ptr(), st))
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        assert torch.isfinite(out).all()
        # the same kernels on the same inputs, only the scratch address differs: bit-identical output
        assert torch.equal(out, ref), (precision, N, starting)


def test_noalloc_refuses_sizes_beyond_its_array():
    f = _noalloc()
    # N = 512 needs far more than the 48 MiB array: refused on the host, nothing launched, no CUDA call
    rc = f(4096, None, 4096, 1, 512, 1, 1e9, _lib.BF16, 1, 4096, None)
    assert rc == _lib.ENOSPACE
    msg = _lib.lib().triattn_last_error_string().decode()
    assert "scratch" in msg and "bytes" in msg
    # invalid arguments are reported like triattn_forward reports them
    assert f(4096, None, 4096, 1, 0, 1, 1e9, _lib.BF16, 1, 4096, None) == _lib.EINVAL
    assert f(4096, None, 4096, 1, 8, 1, 1e9, 7, 1, 4096, None) == _lib.EUNSUPPORTED
