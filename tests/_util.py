"""Shared helpers of the GPU tests: modules built from oracle parameter dicts, random masks with the
reference tests' patterns, and the tolerances of BASELINE.json's north star."""

from __future__ import annotations

import numpy as np
import torch

from boltz_mlx_b200 import TriangleAttention, load_params
from oracle.triattn_ref import metrics

# fp32 mode: max relative error (max|d| / max|ref|) <= 1e-5 against the fp32 reference path.
FP32_MAX_REL = 1e-5
# 16-bit modes (fp32 accumulation): max abs <= 2e-2 and mean abs <= 5e-3 against the fp32 reference.
H16_MAX_ABS = 2e-2
H16_MEAN_ABS = 5e-3


def module(params: dict, starting: bool, precision: str, device="cuda") -> TriangleAttention:
    m = TriangleAttention(128, 32, 4, starting=starting, inf=1e9, precision=precision).to(device)
    return load_params(m, {k: (v.to(device) if v is not None else None) for k, v in params.items()})


def rand_mask(g: torch.Generator, B: int, N: int, pattern: str = "rows_cols") -> torch.Tensor:
    m = (torch.rand(B, N, N, generator=g) > 0.3).float()
    if pattern == "rows_cols" and N > 7:
        m[:, 3, :] = 0.0  # fully masked row
        m[:, :, 5] = 0.0  # masked key column
        m[:, 7, :] = 0.0
    if pattern == "keep_col0":
        m[:, :, 0] = 1.0
    return m


def assert_parity(out, ref, precision: str, name: str = "") -> dict:
    out = out.detach().double().cpu().numpy() if torch.is_tensor(out) else np.asarray(out)
    ref = ref.detach().double().cpu().numpy() if torch.is_tensor(ref) else np.asarray(ref)
    m = metrics(out, ref)
    assert m["finite"], f"{name}: non-finite output"
    if precision == "fp32":
        assert m["max_rel"] <= FP32_MAX_REL, f"{name}: {m}"
    else:
        assert m["max_abs"] <= H16_MAX_ABS and m["mean_abs"] <= H16_MEAN_ABS, f"{name}: {m}"
    return m
