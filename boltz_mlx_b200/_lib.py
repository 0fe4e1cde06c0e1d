"""ctypes binding of libtriattn.so (the C ABI declared in include/triattn.h).

The library is the only compute path: there is no CPU or PyTorch fallback.  If the shared object is
missing, `lib()` raises ImportError; if a CUDA tensor is not supplied, the wrappers raise.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).with_name("libtriattn.so")

OK, EINVAL, EUNSUPPORTED, ECUDA, EDEVICE, ENOSPACE = 0, 1, 2, 3, 4, 5
F32, F16, BF16 = 0, 1, 2
DTYPES = {"fp32": F32, "float32": F32, "fp16": F16, "float16": F16, "f16": F16, "bf16": BF16, "bfloat16": BF16}

EXPORTED = [
    "triattn_version", "triattn_last_error_string", "triattn_device_status", "triattn_packed_weights_bytes",
    "triattn_pack_weights", "triattn_workspace_bytes", "triattn_forward", "triattn_mask_prep",
    "triattn_ln_proj", "triattn_core", "triattn_out_proj", "triattn_mask_prep_v", "triattn_ln_proj_v",
    "triattn_out_proj_v", "triattn_ln_proj_vb", "triattn_out_proj_vb", "triattn_forward_fused",
    "triattn_out_proj_vt", "triattn_peer_alloc", "triattn_peer_free", "triattn_ipc_handle", "triattn_ipc_open",
    "triattn_ipc_close", "triattn_peer_barrier", "triattn_peer_broadcast", "triattn_forward_chunked",
    "triattn_trimul_packed_bytes", "triattn_trimul_pack_weights", "triattn_trimul_workspace_bytes",
    "triattn_trimul_forward", "triattn_trimul_forward_addln", "triattn_forward_fused_tb",
    "triattn_trimul_forward_addln_tb",
]
IPC_HANDLE_BYTES = 64


class TriAttnError(RuntimeError):
    """A libtriattn call returned a non-zero status."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"libtriattn status {code}: {msg}")
        self.code = code


class TriAttnInvalid(TriAttnError, ValueError):
    pass


class TriAttnUnsupported(TriAttnError, NotImplementedError):
    pass


_L = None
_vp, _i, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t


def lib() -> ctypes.CDLL:
    global _L
    if _L is None:
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is not built; run `python -m boltz_mlx_b200.build`")
        L = ctypes.CDLL(str(LIB_PATH))
        L.triattn_version.restype = ctypes.c_char_p
        L.triattn_version.argtypes = []
        L.triattn_last_error_string.restype = ctypes.c_char_p
        L.triattn_last_error_string.argtypes = []
        L.triattn_device_status.argtypes = [ctypes.POINTER(ctypes.c_int), _i]
        L.triattn_packed_weights_bytes.restype = _sz
        L.triattn_packed_weights_bytes.argtypes = [_i]
        L.triattn_pack_weights.argtypes = [_vp] * 9 + [_i, _vp, _sz, _vp]
        L.triattn_workspace_bytes.restype = _sz
        L.triattn_workspace_bytes.argtypes = [_i, _i, _i, _i]
        L.triattn_forward.argtypes = [_vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _vp, _vp, _sz, _vp]
        L.triattn_forward_chunked.argtypes = [_vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _vp, _i, _vp, _sz, _vp]
        L.triattn_forward_fused.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _vp, _i, _vp, _vp, _vp, _i,
                                            _vp, _sz, _vp]
        L.triattn_forward_fused_tb.argtypes = [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _i, _vp, _i, _vp, _vp,
                                               _vp, _i, _vp, _vp, _vp, _sz, _vp]
        L.triattn_mask_prep.argtypes = [_vp, _i, _i, _i, _f, _i, _i, _i, _vp, _sz, _vp]
        L.triattn_ln_proj.argtypes = [_vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]
        L.triattn_core.argtypes = [_i, _i, _i, _i, _i, _vp, _sz, _vp]
        L.triattn_out_proj.argtypes = [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp]
        _l = ctypes.c_int64
        L.triattn_mask_prep_v.argtypes = [_vp, _l, _l, _l, _i, _i, _f, _i, _i, _i, _vp, _sz, _vp]
        L.triattn_ln_proj_v.argtypes = [_vp, _l, _l, _l, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp]
        L.triattn_out_proj_v.argtypes = [_vp, _l, _l, _l, _vp, _l, _l, _l, _vp, _i, _i, _i, _i, _i, _i, _vp, _sz,
                                         _vp]
        L.triattn_ln_proj_vb.argtypes = [_vp, _l, _l, _l, _i, _l, _vp, _i, _i, _i, _i, _i, _vp, _sz, _vp]
        L.triattn_out_proj_vb.argtypes = [_vp, _l, _l, _l, _i, _l, _vp, _l, _l, _l, _i, _l, _vp, _i, _i, _i, _i, _i,
                                          _i, _vp, _sz, _vp]
        L.triattn_out_proj_vt.argtypes = [_vp, _l, _l, _l, _i, _l, _vp, _l, _l, _l, _i, _vp, _vp, _i, _i, _i, _i, _i,
                                          _i, _vp, _sz, _vp]
        L.triattn_peer_alloc.argtypes = [_sz, ctypes.POINTER(_vp)]
        L.triattn_peer_free.argtypes = [_vp]
        L.triattn_ipc_handle.argtypes = [_vp, ctypes.c_char_p]
        L.triattn_ipc_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(_vp)]
        L.triattn_ipc_close.argtypes = [_vp]
        L.triattn_peer_barrier.argtypes = [_vp, _i, _i, ctypes.c_uint32, _vp]
        L.triattn_peer_broadcast.argtypes = [_vp, _i, _i, _sz, _sz, _vp]
        L.triattn_trimul_packed_bytes.restype = _sz
        L.triattn_trimul_packed_bytes.argtypes = [_i]
        L.triattn_trimul_workspace_bytes.restype = _sz
        L.triattn_trimul_workspace_bytes.argtypes = [_i, _i, _i]
        L.triattn_trimul_pack_weights.argtypes = [_vp] * 8 + [_i, _vp, _sz, _vp]
        L.triattn_trimul_forward.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp]
        L.triattn_trimul_forward_addln.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _sz, _vp]
        L.triattn_trimul_forward_addln_tb.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp,
                                                      _vp, _sz, _vp]
        for name in EXPORTED:
            if name not in ("triattn_version", "triattn_last_error_string", "triattn_packed_weights_bytes",
                            "triattn_workspace_bytes", "triattn_trimul_packed_bytes",
                            "triattn_trimul_workspace_bytes"):
                getattr(L, name).restype = ctypes.c_int
        _L = L
    return _L


def check(rc: int) -> None:
    if rc == OK:
        return
    msg = (lib().triattn_last_error_string() or b"").decode(errors="replace")
    if rc == EINVAL or rc == ENOSPACE:
        raise TriAttnInvalid(rc, msg)
    if rc == EUNSUPPORTED:
        raise TriAttnUnsupported(rc, msg)
    raise TriAttnError(rc, msg)


def dtype_code(precision) -> int:
    if isinstance(precision, int):
        return precision
    if isinstance(precision, torch.dtype):
        precision = str(precision).replace("torch.", "")
    try:
        return DTYPES[str(precision).lower()]
    except KeyError:
        raise TriAttnUnsupported(EUNSUPPORTED, f"precision {precision!r}") from None


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def device_status(clear: bool = True) -> int:
    """The device status word (0 = ok; 101..103 = a bounded wait ran out, 105 unaligned
    shared memory, 106 a cross-GPU barrier missed a peer).  Synchronises."""
    v = ctypes.c_int(0)
    check(lib().triattn_device_status(ctypes.byref(v), int(clear)))
    return v.value


def packed_weights_bytes(dtype: int) -> int:
    return int(lib().triattn_packed_weights_bytes(dtype))


def workspace_bytes(B: int, N: int, rows: int, dtype: int) -> int:
    return int(lib().triattn_workspace_bytes(B, N, rows, dtype))


def version() -> str:
    return lib().triattn_version().decode()
