"""CPU: the row-chunked layer's host logic -- chunk sizes chosen by the module and argument checks of
triattn_forward_chunked (no kernel is launched)."""

import pytest

from boltz_mlx_b200 import TriangleAttention, _lib
from boltz_mlx_b200.build import build
from boltz_mlx_b200.layout import workspace_bytes


@pytest.mark.parametrize("dtype", [_lib.F32, _lib.BF16])
@pytest.mark.parametrize("N", [1, 100, 384, 1024, 2048, 3000, 4096, 8192, 16384])
def test_automatic_chunks_fit_the_budget(dtype, N):
    mod = TriangleAttention(precision="fp32" if dtype == _lib.F32 else "bf16")
    rows = mod.chunk_rows(1, N, dtype)
    assert 1 <= rows <= N
    if rows < N:
        assert rows % 128 == 0
        assert workspace_bytes(1, N, rows, dtype) <= mod.max_workspace_bytes or rows == 128
        # the largest such chunk: one more tile no longer fits
        assert rows + 128 >= N or workspace_bytes(1, N, rows + 128, dtype) > mod.max_workspace_bytes
    else:
        assert workspace_bytes(1, N, N, dtype) <= mod.max_workspace_bytes


def test_explicit_chunk_size():
    mod = TriangleAttention(precision="bf16")
    assert mod.chunk_rows(1, 300, _lib.BF16, 100) == 128  # whole 128-row tri-bias blocks on the 16-bit path
    assert mod.chunk_rows(1, 300, _lib.F32, 100) == 100
    assert mod.chunk_rows(1, 100, _lib.BF16, 64) == 100  # one chunk
    with pytest.raises(ValueError):
        mod.chunk_rows(1, 300, _lib.BF16, 0)
    mod.max_workspace_bytes = 0
    assert mod.chunk_rows(1, 1024, _lib.BF16) == 128  # never below one tile


def test_chunked_entry_validates_on_the_host():
    build()
    L = _lib.lib()

    def call(N=300, dtype=_lib.BF16, chunk=128, ws_bytes=1 << 34, z=4096, out=4096):
        return L.triattn_forward_chunked(z, None, 256 * 16, 1, N, 1, 1e9, dtype, 1, out, chunk, 256 * 4096, ws_bytes,
                                         None)

    assert call(chunk=0) == _lib.EINVAL
    assert call(chunk=100) == _lib.EINVAL  # 16-bit chunks are whole 128-row tiles
    assert call(z=4096 + 4) == _lib.EINVAL
    assert call(ws_bytes=workspace_bytes(1, 300, 128, _lib.BF16) - 1) == _lib.ENOSPACE
    assert call(N=0) == _lib.EINVAL
