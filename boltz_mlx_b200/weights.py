"""Converted-checkpoint loading for the triangle-attention modules (the reference keeps PyTorch
qualified names in its safetensors files: boltz_mlx/weights.py:18-35, boltz2_{name}.safetensors).

The safetensors container is read and written here directly (the `safetensors` package is not a
dependency): an 8-byte little-endian header length, a JSON header mapping every tensor name to
{"dtype", "shape", "data_offsets": [begin, end]} (offsets into the byte buffer that follows the
header), optionally "__metadata__", then the raw little-endian data.

    tensors = read_safetensors("boltz2_conf.safetensors")
    start = load_module(TriangleAttention(starting=True), "pairformer_module.layers.0.tri_att_start", tensors)
    start, end = load_pairformer_triatt(tensors, layer=0, precision="bf16")
"""

from __future__ import annotations

import json
import os
import struct
from pathlib import Path
from typing import Optional, Union

import numpy as np
import torch

from .triangle_attention import TriangleAttention

_DTYPES = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool,
}
_NAMES = {v: k for k, v in _DTYPES.items()}


def read_safetensors(path: Union[str, os.PathLike]) -> dict:
    """All tensors of a safetensors file, as CPU torch tensors (copies; the file is not kept open)."""
    data = Path(path).read_bytes()
    if len(data) < 8:
        raise ValueError(f"{path}: not a safetensors file (shorter than its header length)")
    (n,) = struct.unpack("<Q", data[:8])
    if 8 + n > len(data):
        raise ValueError(f"{path}: header length {n} exceeds the file")
    header = json.loads(data[8:8 + n].decode("utf-8"))
    buf = memoryview(data)[8 + n:]
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = _DTYPES.get(info["dtype"])
        if dt is None:
            raise ValueError(f"{path}: tensor {name}: unsupported dtype {info['dtype']}")
        b0, b1 = info["data_offsets"]
        shape = tuple(info["shape"])
        esize = torch.empty((), dtype=dt).element_size()
        if b1 - b0 != int(np.prod(shape, dtype=np.int64)) * esize or b1 > len(buf):
            raise ValueError(f"{path}: tensor {name}: data_offsets {b0}..{b1} do not match shape {shape}")
        if b1 == b0:
            out[name] = torch.empty(shape, dtype=dt)
            continue
        raw = torch.frombuffer(bytearray(buf[b0:b1]), dtype=torch.uint8)
        out[name] = raw.view(dt).reshape(shape)
    return out


def write_safetensors(path: Union[str, os.PathLike], tensors: dict, metadata: Optional[dict] = None) -> None:
    """Write tensors (any device; stored contiguous, little-endian) in the safetensors layout."""
    header, chunks, off = {}, [], 0
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        if t.dtype not in _NAMES:
            raise ValueError(f"tensor {name}: unsupported dtype {t.dtype}")
        b = t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        chunks.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hb += b" " * (-len(hb) % 8)  # the data buffer starts 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for b in chunks:
            f.write(b)


def subtree(tensors: dict, prefix: str) -> dict:
    """Tensors under `prefix`, with names relative to it (weights.py:22-24)."""
    p = prefix.rstrip(".") + "."
    return {k[len(p):]: v for k, v in tensors.items() if k.startswith(p)}


def load_module(module: torch.nn.Module, prefix: str, tensors: Union[dict, str, os.PathLike],
                strict: bool = True) -> torch.nn.Module:
    """Load the tensors under `prefix` into `module` (weights.py:27-35): with `strict`, missing or
    unexpected names raise ValueError naming them; values are cast to each parameter's dtype and
    device."""
    if not isinstance(tensors, dict):
        tensors = read_safetensors(tensors)
    w = subtree(tensors, prefix)
    ours = dict(module.named_parameters())
    if strict:
        missing, extra = set(ours) - set(w), set(w) - set(ours)
        if missing or extra:
            raise ValueError(f"{prefix}: missing={sorted(missing)[:10]} unexpected={sorted(extra)[:10]}")
    with torch.no_grad():
        for name, p in ours.items():
            if name in w:
                v = w[name]
                if tuple(v.shape) != tuple(p.shape):
                    raise ValueError(f"{prefix}.{name}: shape {tuple(v.shape)} != {tuple(p.shape)}")
                p.copy_(v.to(device=p.device, dtype=p.dtype))
    return module


def load_pairformer_triatt(tensors: Union[dict, str, os.PathLike], layer: int, *,
                           stack: str = "pairformer_module", precision: Optional[str] = None,
                           device: Union[str, torch.device] = "cuda", inf: float = 1e9):
    """(start, end) TriangleAttention modules of pairformer layer `layer` of `stack`
    (`{stack}.layers.{layer}.tri_att_{start,end}.*`, tests/test_trunk_layers.py:96-97)."""
    if not isinstance(tensors, dict):
        tensors = read_safetensors(tensors)
    mods = []
    for starting, tag in ((True, "tri_att_start"), (False, "tri_att_end")):
        m = TriangleAttention(128, 32, 4, starting=starting, inf=inf, precision=precision).to(device)
        mods.append(load_module(m, f"{stack}.layers.{layer}.{tag}", tensors))
    return tuple(mods)
