"""CPU oracle for the pairformer triangle multiplication (outgoing / incoming edges, forward).

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module: only `tests/` and
`bench.py`'s CPU-baseline arm use it, as the checker or the timed CPU baseline.

Parity status: UNPINNED against the reference's own outputs (the reference runs on Apple MLX, which
is not installable here, and no dumps of this module are committed).  This file restates the
reference's fp32 ops path and is cross-checked against an independently written float64 loop form
(`trimul_np64`) in tests/test_trimul_oracle.py.

What it restates (file:line inside the reference project):
  boltz_mlx/layers/triangular_mult.py:13-21    parameters: norm_in (LayerNorm 128, eps 1e-5), p_in / g_in
                                               Linear(128 -> 256, no bias), norm_out (LayerNorm 128,
                                               mlx default eps 1e-5), p_out / g_out Linear(128 -> 128, no bias)
  triangular_mult.py:28,33-37                  xn = norm_in(x); h = xn @ [p_in | g_in | g_out]^T
  triangular_mult.py:38-41                     x = p * sigmoid(g) * mask[..., None]; a, b = x[..., :D], x[..., D:]
  triangular_mult.py:43-47                     outgoing: o[i,j,d] = sum_k a[i,k,d] b[j,k,d]
                                               incoming: o[i,j,d] = sum_k a[k,i,d] b[k,j,d]
  triangular_mult.py:49                        y = p_out(norm_out(o)) * sigmoid(g_out)
The module returns the UPDATE y; the pairformer adds the residual (pairformer.py z += tri_mul_out(z)).
"""

from __future__ import annotations

from typing import Optional

import numpy as np
import torch

D = 128
LN_EPS = 1e-5

PARAM_SHAPES = {
    "in_w": (D,), "in_b": (D,),          # norm_in
    "p_in": (2 * D, D), "g_in": (2 * D, D),
    "out_w": (D,), "out_b": (D,),        # norm_out
    "p_out": (D, D), "g_out": (D, D),
}
# reference parameter names (checkpoint keys under ...tri_mul_{out,in}.)
REF_NAMES = {
    "in_w": "norm_in.weight", "in_b": "norm_in.bias", "p_in": "p_in.weight", "g_in": "g_in.weight",
    "out_w": "norm_out.weight", "out_b": "norm_out.bias", "p_out": "p_out.weight", "g_out": "g_out.weight",
}


def make_params(seed: int, *, ln_identity: bool = False) -> dict:
    """Seeded synthetic parameters: linears ~ N(0, 1/128); LayerNorm affine ~ 1 + 0.1 N(0,1) / 0.1 N(0,1)
    (identity with ln_identity)."""
    g = torch.Generator().manual_seed(seed)
    p = {}
    for k, shp in PARAM_SHAPES.items():
        if k in ("in_w", "out_w"):
            p[k] = torch.ones(shp) if ln_identity else 1.0 + 0.1 * torch.randn(shp, generator=g)
        elif k in ("in_b", "out_b"):
            p[k] = torch.zeros(shp) if ln_identity else 0.1 * torch.randn(shp, generator=g)
        else:
            p[k] = torch.randn(shp, generator=g) / np.sqrt(D)
    return p


def _layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    mean = x.mean(-1, keepdim=True)
    var = ((x - mean) ** 2).mean(-1, keepdim=True)
    return (x - mean) * torch.rsqrt(var + LN_EPS) * w + b


def trimul_ref(z: torch.Tensor, mask: Optional[torch.Tensor], params: dict, *, outgoing: bool = True,
               dtype: torch.dtype = torch.float32, channel_block: int = 32) -> torch.Tensor:
    """y = TriangleMultiplication{Outgoing,Incoming}(z, mask) on the CPU in `dtype`.  z [B, N, N, 128],
    mask [B, N, N] or None (ones).  Returns the update y [B, N, N, 128].  The contraction runs over
    blocks of channels (channels are independent, triangular_mult.py:60-61) to bound memory."""
    x = z.to(dtype)
    B, N = x.shape[0], x.shape[1]
    m = torch.ones(B, N, N, dtype=dtype) if mask is None else mask.to(dtype)
    P = {k: v.to(dtype) for k, v in params.items()}
    xn = _layer_norm(x, P["in_w"], P["in_b"])
    w = torch.cat([P["p_in"], P["g_in"], P["g_out"]], 0)  # [640, 128]
    g_out = xn @ P["g_out"].T
    o = torch.empty(B, N, N, D, dtype=dtype)
    for c0 in range(0, D, channel_block):
        c1 = min(D, c0 + channel_block)
        rows = list(range(c0, c1)) + list(range(D + c0, D + c1))  # a and b channels of the block
        pw, gw = P["p_in"][rows], P["g_in"][rows]
        h = (xn @ pw.T) * torch.sigmoid(xn @ gw.T) * m[..., None]  # [B, N, N, 2n]
        n = c1 - c0
        a = h[..., :n].permute(0, 3, 1, 2)  # [B, n, N(i), N(k)]
        b = h[..., n:].permute(0, 3, 1, 2)
        if outgoing:
            oc = a @ b.transpose(-1, -2)    # sum_k a[i,k] b[j,k]
        else:
            oc = a.transpose(-1, -2) @ b    # sum_k a[k,i] b[k,j]
        o[..., c0:c1] = oc.permute(0, 2, 3, 1)
    del w
    return (_layer_norm(o, P["out_w"], P["out_b"]) @ P["p_out"].T) * torch.sigmoid(g_out)


def trimul_np64(z: np.ndarray, mask: Optional[np.ndarray], params: dict, *, outgoing: bool = True) -> np.ndarray:
    """Independent float64 formulation (explicit einsums) for cross-checking trimul_ref."""
    x = np.asarray(z, np.float64)
    B, N = x.shape[0], x.shape[1]
    m = np.ones((B, N, N)) if mask is None else np.asarray(mask, np.float64)
    P = {k: np.asarray(v, np.float64) for k, v in params.items()}

    def ln(t, w, b):
        mu = t.mean(-1, keepdims=True)
        sd = np.sqrt(((t - mu) ** 2).mean(-1, keepdims=True) + LN_EPS)
        return (t - mu) / sd * w + b

    xn = ln(x, P["in_w"], P["in_b"])
    p = np.einsum("bijc,oc->bijo", xn, P["p_in"])
    g = np.einsum("bijc,oc->bijo", xn, P["g_in"])
    ab = p / (1.0 + np.exp(-g)) * m[..., None]
    a, b = ab[..., :D], ab[..., D:]
    o = np.einsum("bikd,bjkd->bijd", a, b) if outgoing else np.einsum("bkid,bkjd->bijd", a, b)
    go = np.einsum("bijc,oc->bijo", xn, P["g_out"])
    return np.einsum("bijc,oc->bijo", ln(o, P["out_w"], P["out_b"]), P["p_out"]) / (1.0 + np.exp(-go))
