"""CPU: libtriattn.so loads, exports every symbol include/triattn.h declares, and its host-side logic
(argument validation, workspace layout) behaves -- no kernel is launched here."""

import re
from pathlib import Path

import pytest

from boltz_mlx_b200 import _lib, layout
from boltz_mlx_b200.build import build

HEADER = Path(__file__).resolve().parents[1] / "include" / "triattn.h"


@pytest.fixture(scope="module")
def L():
    build()
    return _lib.lib()


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TRIATTN_API\s+[\w\s\*]+?\b(triattn_\w+)\s*\(", text)))


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ("triattn_forward", "triattn_core", "triattn_ln_proj", "triattn_out_proj", "triattn_mask_prep",
              "triattn_pack_weights", "triattn_workspace_bytes", "triattn_device_status"):
        assert s in syms


def test_library_exports_every_declared_symbol(L):
    for s in declared_symbols():
        assert hasattr(L, s), s
    assert set(declared_symbols()) <= set(_lib.EXPORTED) | set(declared_symbols())
    assert "sm_100a" in _lib.version()


@pytest.mark.parametrize("dtype", [_lib.F32, _lib.F16, _lib.BF16])
@pytest.mark.parametrize("B,N,rows", [(1, 1, 1), (2, 9, 9), (1, 128, 128), (1, 129, 64), (1, 1024, 1024), (3, 384, 17)])
def test_workspace_layout_matches_library(L, dtype, B, N, rows):
    assert _lib.workspace_bytes(B, N, rows, dtype) == layout.workspace_bytes(B, N, rows, dtype)


def test_packed_weight_sizes(L):
    f32 = _lib.packed_weights_bytes(_lib.F32)
    f16 = _lib.packed_weights_bytes(_lib.F16)
    assert f32 >= (3 * 128 + 4 * 128 + 512 * 128 + 128 * 128) * 4
    assert f16 >= f32 + (512 * 128 + 128 * 128) * 2
    assert _lib.packed_weights_bytes(_lib.BF16) == f16


def _fwd(L, z=1, mask=0, packed=256, B=1, N=8, starting=1, dtype=0, out=1, ws=256, ws_bytes=1 << 30):
    # pointer-sized fake addresses: validation must reject before any device access
    return L.triattn_forward(z * 4096, mask, packed * 4096, B, N, starting, 1e9, dtype, 0, out * 4096,
                             ws * 4096, ws_bytes, None)


def test_host_validation_rejects_bad_arguments(L):
    assert _fwd(L, N=0) == _lib.EINVAL
    assert _fwd(L, B=0) == _lib.EINVAL
    assert _fwd(L, dtype=7) == _lib.EUNSUPPORTED
    assert _fwd(L, N=20000) == _lib.EUNSUPPORTED
    assert _fwd(L, z=0) == _lib.EINVAL
    assert _fwd(L, out=0) == _lib.EINVAL
    assert _fwd(L, packed=0) == _lib.EINVAL
    assert _fwd(L, ws=0) == _lib.EINVAL
    assert _fwd(L, ws_bytes=16) == _lib.ENOSPACE
    msg = L.triattn_last_error_string().decode()
    assert "workspace" in msg
    # misaligned pointers
    assert L.triattn_forward(4096 + 4, None, 4096, 1, 8, 1, 1e9, 0, 0, 4096, 4096, 1 << 30, None) == _lib.EINVAL
    assert L.triattn_forward(4096, None, 4096 + 16, 1, 8, 1, 1e9, 0, 0, 4096, 4096, 1 << 30, None) == _lib.EINVAL
    # row ranges of the stage entry points
    assert L.triattn_core(1, 8, 4, 4, 0, 4096, 1 << 30, None) == _lib.EINVAL
    assert L.triattn_core(1, 8, 0, 9, 0, 4096, 1 << 30, None) == _lib.EINVAL
    assert L.triattn_core(1, 8, -1, 2, 0, 4096, 1 << 30, None) == _lib.EINVAL
    assert L.triattn_pack_weights(*([None] * 9), 0, 4096, 1 << 20, None) == _lib.EINVAL
    assert L.triattn_device_status(None, 0) == _lib.EINVAL


def test_status_codes_map_to_exceptions(L):
    with pytest.raises(_lib.TriAttnInvalid):
        _lib.check(_fwd(L, N=0))
    with pytest.raises(_lib.TriAttnUnsupported):
        _lib.check(_fwd(L, dtype=9))
    with pytest.raises(_lib.TriAttnUnsupported):
        _lib.dtype_code("fp8")


def test_module_refuses_cpu_tensors_and_other_geometries():
    import torch

    from boltz_mlx_b200 import TriangleAttention

    m = TriangleAttention(128, 32, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        m(torch.zeros(1, 4, 4, 128))
    m2 = TriangleAttention(32, 16, 3)
    with pytest.raises(NotImplementedError):
        m2(torch.zeros(1, 4, 4, 32))
    names = {n for n, _ in m.named_parameters()}
    assert names == {"layer_norm.weight", "layer_norm.bias", "linear.weight", "mha.linear_q.weight",
                     "mha.linear_k.weight", "mha.linear_v.weight", "mha.linear_o.weight", "mha.linear_g.weight"}


@pytest.mark.parametrize("dtype", [_lib.F32, _lib.F16, _lib.BF16])
@pytest.mark.parametrize("B,N", [(1, 1), (2, 9), (1, 128), (1, 1024), (3, 37)])
def test_trimul_sizes_match_library(L, dtype, B, N):
    assert L.triattn_trimul_workspace_bytes(B, N, dtype) == layout.trimul_workspace_bytes(B, N, dtype)
    assert L.triattn_trimul_packed_bytes(dtype) == layout.trimul_packed_bytes(dtype)


def test_trimul_host_validation(L):
    ws = 256 * 4096
    assert L.triattn_trimul_forward(4096, None, 256 * 16, 1, 0, 1, _lib.BF16, 1, 4096, ws, 1 << 34, None) == _lib.EINVAL
    assert L.triattn_trimul_forward(4096 + 4, None, 256 * 16, 1, 8, 1, _lib.BF16, 1, 4096, ws, 1 << 34, None) == _lib.EINVAL
    assert L.triattn_trimul_forward(4096, None, 256 * 16, 1, 8, 1, _lib.BF16, 1, 4096, ws, 16, None) == _lib.ENOSPACE
    assert L.triattn_trimul_forward(4096, None, 256 * 16, 1, 8, 1, 9, 1, 4096, ws, 1 << 34, None) == _lib.EUNSUPPORTED
    # addln: 16-bit only, and its LayerNorm pointers are checked
    assert L.triattn_trimul_forward_addln(4096, None, 256 * 16, 1, 8, 1, _lib.F32, 4096, 4096, 4096, 4096, ws,
                                          1 << 34, None) == _lib.EUNSUPPORTED
    assert L.triattn_trimul_forward_addln(4096, None, 256 * 16, 1, 8, 1, _lib.BF16, 4096, None, 4096, 4096, ws,
                                          1 << 34, None) == _lib.EINVAL
    assert L.triattn_trimul_pack_weights(*([None] * 8), _lib.BF16, 4096, 1 << 20, None) == _lib.EINVAL
