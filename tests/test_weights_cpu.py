"""CPU: the converted-checkpoint path (boltz_mlx/weights.py:18-35) -- the safetensors container read
and written by boltz_mlx_b200.weights, strict loading of the reference's qualified names into the
modules, and its errors."""

import json
import struct

import pytest
import torch

from boltz_mlx_b200 import TriangleAttention
from boltz_mlx_b200.weights import load_module, load_pairformer_triatt, read_safetensors, subtree, write_safetensors
from oracle.triattn_ref import PARAM_SHAPES


def test_round_trip_dtypes(tmp_path):
    g = torch.Generator().manual_seed(0)
    ts = {
        "a.f32": torch.randn(3, 5, generator=g),
        "a.f16": torch.randn(7, generator=g).half(),
        "b.bf16": torch.randn(2, 2, 2, generator=g).bfloat16(),
        "c.i64": torch.arange(11, dtype=torch.int64),
        "d.empty": torch.empty(0, 4),
        "e.scalar": torch.tensor(3.5),
    }
    p = tmp_path / "x.safetensors"
    write_safetensors(p, ts, metadata={"format": "pt"})
    back = read_safetensors(p)
    assert set(back) == set(ts)
    for k, v in ts.items():
        assert back[k].dtype == v.dtype and back[k].shape == v.shape and torch.equal(back[k], v), k
    # container layout: u64 header length, JSON header padded to 8 bytes, contiguous data offsets
    raw = p.read_bytes()
    (n,) = struct.unpack("<Q", raw[:8])
    assert n % 8 == 0
    hdr = json.loads(raw[8:8 + n])
    assert hdr["__metadata__"] == {"format": "pt"}
    spans = sorted(v["data_offsets"] for k, v in hdr.items() if k != "__metadata__")
    assert spans[0][0] == 0 and all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert spans[-1][1] == len(raw) - 8 - n


def _ckpt(layer=0, stack="pairformer_module", drop=None, extra=None):
    g = torch.Generator().manual_seed(layer)
    names = {"w_q": "mha.linear_q.weight", "w_k": "mha.linear_k.weight", "w_v": "mha.linear_v.weight",
             "w_g": "mha.linear_g.weight", "w_o": "mha.linear_o.weight", "w_b": "linear.weight"}
    ts = {}
    for tag in ("tri_att_start", "tri_att_end"):
        pre = f"{stack}.layers.{layer}.{tag}."
        for key, name in names.items():
            ts[pre + name] = torch.randn(PARAM_SHAPES[key], generator=g)
        ts[pre + "layer_norm.weight"] = 1 + 0.1 * torch.randn(128, generator=g)
        ts[pre + "layer_norm.bias"] = 0.1 * torch.randn(128, generator=g)
    ts["other_module.weight"] = torch.zeros(3)
    if drop:
        del ts[drop]
    if extra:
        ts[extra] = torch.zeros(1)
    return ts


def test_strict_load_reference_names(tmp_path):
    ts = _ckpt(layer=5)
    p = tmp_path / "boltz2_conf.safetensors"
    write_safetensors(p, ts)
    start, end = load_pairformer_triatt(p, 5, device="cpu")
    assert start.starting and not end.starting
    for tag, m in (("tri_att_start", start), ("tri_att_end", end)):
        sub = subtree(ts, f"pairformer_module.layers.5.{tag}")
        for name, prm in m.named_parameters():
            assert torch.equal(prm.detach(), sub[name]), (tag, name)


def test_strict_load_errors():
    m = TriangleAttention(starting=True)
    with pytest.raises(ValueError, match="missing="):
        load_module(m, "pairformer_module.layers.0.tri_att_start",
                    _ckpt(drop="pairformer_module.layers.0.tri_att_start.mha.linear_o.weight"))
    with pytest.raises(ValueError, match="unexpected="):
        load_module(m, "pairformer_module.layers.0.tri_att_start",
                    _ckpt(extra="pairformer_module.layers.0.tri_att_start.mha.linear_o.bias"))
    bad = _ckpt()
    bad["pairformer_module.layers.0.tri_att_start.linear.weight"] = torch.zeros(5, 128)
    with pytest.raises(ValueError, match="shape"):
        load_module(m, "pairformer_module.layers.0.tri_att_start", bad)
    # non-strict: missing names keep the module's values
    ok = load_module(TriangleAttention(starting=True), "pairformer_module.layers.0.tri_att_start",
                     _ckpt(drop="pairformer_module.layers.0.tri_att_start.linear.weight"), strict=False)
    assert ok.linear.weight.shape == (4, 128)


def test_truncated_file_rejected(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(ValueError):
        read_safetensors(p)
