"""CPU oracle for the pairformer triangle attention (starting / ending node, forward).

TEST INFRASTRUCTURE ONLY.  Nothing in the product path imports this module: only
`tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline / reference arm
use it, and only as the checker or the timed CPU baseline.

Parity status: UNPINNED against the reference's own outputs.  The reference
(jackryan225/boltz-mlx) runs on Apple MLX, which is not installable in this
container, and its parity dumps (data/prot117/ref/modules/*.npz) and converted
weights are not committed.  This file restates the reference's fp32 ops path
and is cross-checked against a second, independently written float64
formulation (`tri_attention_np64`) and against the committed golden fixtures
in tests/golden/ (generated from this oracle by tests/golden/make_golden.py).

What it restates (file:line inside the reference project):
  boltz_mlx/layers/triangular_attention/attention.py:37-38   default mask = ones
  attention.py:40-42                                          ending node: swap axes of x and mask
  attention.py:47 / primitives.py:16-17                       LayerNorm, eps 1e-5, fp32 statistics
  attention.py:49-53,69                                       fused projection W = [q|k|v|g|linear], h = xn @ W^T
  attention.py:80-83                                          q,k,v -> [B*I, H, J, C] (channel = head*C + d); g = h[..., 3HC:4HC]
  attention.py:84                                             tri_bias[b,h,q,k] = h[b,q,k,4HC+h]
  attention.py:85                                             mask_bias[b,i,k] = inf * (mask[b,i,k] - 1)
  attention.py:86-87                                          softmax((q*C^-1/2) k^T + (tri_bias + mask_bias)) v
  attention.py:89                                             y = linear_o(o * sigmoid(g))
  attention.py:91-92                                          swap back for the ending node
  attention.py:55-68                                          row chunking (identical math; used here to bound memory)
The module returns the UPDATE y; the caller adds the residual (pairformer.py:86-87).

Optional gate bias: the reference's linear_g has no bias (primitives.py:38).  The
benchmark configurations draw a gate bias of 1.0; `params["g_b"]` (None by
default) carries it, in the oracle and in the CUDA path alike.
"""

from __future__ import annotations

import math
from typing import Optional

import numpy as np
import torch

C_IN, HEADS, C_HEAD = 128, 4, 32
HC = HEADS * C_HEAD
LN_EPS = 1e-5
DEFAULT_INF = 1e9

PARAM_SHAPES = {
    "ln_w": (C_IN,),
    "ln_b": (C_IN,),
    "w_q": (HC, C_IN),
    "w_k": (HC, C_IN),
    "w_v": (HC, C_IN),
    "w_g": (HC, C_IN),
    "w_b": (HEADS, C_IN),  # the module's `linear` (tri-bias projection)
    "w_o": (C_IN, HC),
}


def make_params(seed: int, *, gate_bias: Optional[float] = None, ln_identity: bool = True,
                scale: Optional[float] = None) -> dict:
    """Seeded synthetic weights in the reference's [out, in] Linear layout.

    Linears ~ N(0, 1/fan_in) (fan_in = 128 for every linear here) unless `scale` overrides the
    standard deviation; LayerNorm gamma=1 / beta=0 when `ln_identity` (else N(1,0.1)/N(0,0.1))."""
    g = torch.Generator().manual_seed(seed)
    std = (1.0 / C_IN) ** 0.5 if scale is None else scale
    p = {}
    for name in ("w_q", "w_k", "w_v", "w_g", "w_b", "w_o"):
        p[name] = torch.randn(PARAM_SHAPES[name], generator=g, dtype=torch.float32) * std
    if ln_identity:
        p["ln_w"] = torch.ones(C_IN)
        p["ln_b"] = torch.zeros(C_IN)
    else:
        p["ln_w"] = 1.0 + 0.1 * torch.randn(C_IN, generator=g)
        p["ln_b"] = 0.1 * torch.randn(C_IN, generator=g)
    p["g_b"] = None if gate_bias is None else torch.full((HC,), float(gate_bias))
    return p


def _layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    mean = x.mean(-1, keepdim=True)
    var = ((x - mean) ** 2).mean(-1, keepdim=True)
    return (x - mean) * torch.rsqrt(var + LN_EPS) * w + b


def tri_attention_ref(z: torch.Tensor, mask: Optional[torch.Tensor], params: dict, *, starting: bool = True,
                      inf: float = DEFAULT_INF, dtype: torch.dtype = torch.float32,
                      chunk_rows: Optional[int] = None, rows: Optional[tuple] = None,
                      row_ids: Optional[list] = None) -> torch.Tensor:
    """y = TriangleAttention(z, mask) on the CPU in `dtype` (float32 = the reference's fp32 path,
    float64 = the error-budget reference).  z: [B, N, N, 128]; mask: [B, N, N] or None.
    Returns the update y [B, N, N, 128] in z's orientation.

    rows=(r0, r1): compute only attention rows r0..r1-1 (rows are independent once the tri bias of
    all rows is known, attention.py:55-68) and return them in ATTENTION orientation,
    [B, r1-r0, N, 128] (for the ending node attention row a is column a of z).
    row_ids=[a0, a1, ...]: the same for an arbitrary list of attention rows (the LayerNorm and the tri
    bias are computed once), [B, len(row_ids), N, 128] in the listed order."""
    if row_ids is not None:
        x = z.to(dtype)
        m = torch.ones(x.shape[:-1], dtype=dtype) if mask is None else mask.to(dtype)
        if not starting:
            x = x.transpose(-2, -3)
            m = m.transpose(-1, -2)
        P = {k: (v.to(dtype) if v is not None else None) for k, v in params.items()}
        xn = _layer_norm(x, P["ln_w"], P["ln_b"])
        tri_bias = (xn @ P["w_b"].T).permute(0, 3, 1, 2)  # [B, H, Q, K] from ALL rows
        out = [_rows_attention(xn[:, a:a + 1], m[:, a:a + 1], tri_bias, P, inf, dtype) for a in row_ids]
        return torch.cat(out, 1)
    x = z.to(dtype)
    if mask is None:
        mask = torch.ones(x.shape[:-1], dtype=dtype)
    mask = mask.to(dtype)
    if not starting:
        x = x.transpose(-2, -3)
        mask = mask.transpose(-1, -2)
    P = {k: (v.to(dtype) if v is not None else None) for k, v in params.items()}
    xn = _layer_norm(x, P["ln_w"], P["ln_b"])
    w = torch.cat([P["w_q"], P["w_k"], P["w_v"], P["w_g"], P["w_b"]], 0)  # [516, 128]
    B, I, J = xn.shape[:3]
    # tri bias from ALL rows (shared by every row chunk, attention.py:55-58)
    tri_bias = (xn @ w[4 * HC:].T).permute(0, 3, 1, 2)  # [B, H, Q, K]
    wq = w[: 4 * HC]
    scale = C_HEAD ** -0.5
    r_begin, r_end = (0, I) if rows is None else rows
    step = (r_end - r_begin) if chunk_rows is None else chunk_rows
    outs = []
    for i0 in range(r_begin, r_end, step):
        xc = xn[:, i0:min(i0 + step, r_end)]
        Ic = xc.shape[1]
        h = xc @ wq.T  # [B, Ic, J, 512]
        q = h[..., :HC].reshape(B * Ic, J, HEADS, C_HEAD).permute(0, 2, 1, 3)
        k = h[..., HC:2 * HC].reshape(B * Ic, J, HEADS, C_HEAD).permute(0, 2, 1, 3)
        v = h[..., 2 * HC:3 * HC].reshape(B * Ic, J, HEADS, C_HEAD).permute(0, 2, 1, 3)
        g = h[..., 3 * HC:4 * HC]
        if P.get("g_b") is not None:
            g = g + P["g_b"]
        mask_bias = (inf * (mask[:, i0:i0 + Ic] - 1))[:, :, None, None, :]  # [B, Ic, 1, 1, K]
        bias = (tri_bias[:, None] + mask_bias).reshape(B * Ic, HEADS, J, J)
        a = (q * scale) @ k.transpose(-1, -2) + bias
        if dtype != torch.float32:
            # keep the reference's fp32 rounding of masked logits (-1e9 + x lands on the fp32 grid),
            # which makes a fully masked row uniform over all keys
            masked = (mask_bias != 0).expand(B, Ic, HEADS, J, J).reshape(a.shape)
            a = torch.where(masked, a.float().to(dtype), a)
        a = torch.softmax(a, dim=-1)
        o = (a @ v).permute(0, 2, 1, 3).reshape(B, Ic, J, HC)
        outs.append((o * torch.sigmoid(g)) @ P["w_o"].T)
    y = torch.cat(outs, 1)
    if rows is not None:
        return y
    if not starting:
        y = y.transpose(-2, -3)
    return y


def _rows_attention(xc: torch.Tensor, mc: torch.Tensor, tri_bias: torch.Tensor, P: dict, inf: float,
                    dtype: torch.dtype) -> torch.Tensor:
    """Attention rows of LayerNorm output xc [B, Ic, J, 128] with mask rows mc [B, Ic, K] and the tri bias
    of all rows [B, H, Q, K] (attention.py:80-89, the same steps as the chunk loop above)."""
    B, Ic, J = xc.shape[:3]
    wq = torch.cat([P["w_q"], P["w_k"], P["w_v"], P["w_g"]], 0)
    h = xc @ wq.T
    q = h[..., :HC].reshape(B * Ic, J, HEADS, C_HEAD).permute(0, 2, 1, 3)
    k = h[..., HC:2 * HC].reshape(B * Ic, J, HEADS, C_HEAD).permute(0, 2, 1, 3)
    v = h[..., 2 * HC:3 * HC].reshape(B * Ic, J, HEADS, C_HEAD).permute(0, 2, 1, 3)
    g = h[..., 3 * HC:4 * HC]
    if P.get("g_b") is not None:
        g = g + P["g_b"]
    mask_bias = (inf * (mc - 1))[:, :, None, None, :]
    bias = (tri_bias[:, None] + mask_bias).reshape(B * Ic, HEADS, J, J)
    a = (q * C_HEAD ** -0.5) @ k.transpose(-1, -2) + bias
    if dtype != torch.float32:
        masked = (mask_bias != 0).expand(B, Ic, HEADS, J, J).reshape(a.shape)
        a = torch.where(masked, a.float().to(dtype), a)
    a = torch.softmax(a, dim=-1)
    o = (a @ v).permute(0, 2, 1, 3).reshape(B, Ic, J, HC)
    return (o * torch.sigmoid(g)) @ P["w_o"].T


def tri_attention_np64(z: np.ndarray, mask: Optional[np.ndarray], params: dict, *, starting: bool = True,
                       inf: float = DEFAULT_INF) -> np.ndarray:
    """Second, independent float64 formulation (numpy, per-head einsum, explicit max-shifted softmax).

    Follows the upstream add order of primitives.py:60-64 (scores, then + mask_bias, then + tri_bias)
    rather than attention.py's pre-summed bias; in float64 the two agree to rounding."""
    x = np.asarray(z, np.float64)
    B, N1, N2, _ = x.shape
    m = np.ones((B, N1, N2)) if mask is None else np.asarray(mask, np.float64)
    if not starting:
        x = np.swapaxes(x, 1, 2)
        m = np.swapaxes(m, 1, 2)
    P = {k: (None if v is None else np.asarray(v, np.float64)) for k, v in params.items()}
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    xn = (x - mu) / np.sqrt(var + LN_EPS) * P["ln_w"] + P["ln_b"]
    tri = np.einsum("bqkc,hc->bhqk", xn, P["w_b"])
    out = np.zeros(x.shape[:3] + (HC,))
    for hd in range(HEADS):
        sl = slice(hd * C_HEAD, (hd + 1) * C_HEAD)
        q = np.einsum("bijc,dc->bijd", xn, P["w_q"][sl]) / math.sqrt(C_HEAD)
        k = np.einsum("bijc,dc->bijd", xn, P["w_k"][sl])
        v = np.einsum("bijc,dc->bijd", xn, P["w_v"][sl])
        s = np.einsum("bijd,bikd->bijk", q, k)
        mb = np.broadcast_to(inf * (m[:, :, None, :] - 1.0), s.shape)
        s = s + mb
        s = s + tri[:, hd][:, None, :, :]
        # The reference adds the mask bias in fp32: a masked logit -1e9 + x rounds onto the fp32 grid
        # (ulp 64 at 1e9), so a fully masked row becomes uniform over all keys.  Model that rounding.
        s = np.where(mb != 0, s.astype(np.float32).astype(np.float64), s)
        s = s - s.max(-1, keepdims=True)
        e = np.exp(s)
        a = e / e.sum(-1, keepdims=True)
        out[..., sl] = np.einsum("bijk,bikd->bijd", a, v)
    g = np.einsum("bijc,dc->bijd", xn, P["w_g"])
    if P.get("g_b") is not None:
        g = g + P["g_b"]
    y = (out / (1.0 + np.exp(-g))) @ P["w_o"].T
    if not starting:
        y = np.swapaxes(y, 1, 2)
    return y


def metrics(ours, ref, mask=None) -> dict:
    """The reference's parity metrics (boltz_mlx/compare.py:14-33): max_abs, max_rel = max|d| / max|ref|,
    mean_abs, cos; all in float64."""
    a = np.asarray(ours, np.float64)
    b = np.asarray(ref, np.float64)
    if a.shape != b.shape:
        raise ValueError(f"shape mismatch {a.shape} vs {b.shape}")
    if mask is not None:
        msk = np.broadcast_to(np.asarray(mask).astype(bool), a.shape)
        a, b = a[msk], b[msk]
    d = np.abs(a - b)
    scale = max(float(np.abs(b).max(initial=0.0)), 1e-12)
    den = float(np.linalg.norm(a) * np.linalg.norm(b))
    cos = float(a.ravel() @ b.ravel() / den) if den > 0 else (1.0 if d.max(initial=0) == 0 else 0.0)
    return {"max_abs": float(d.max(initial=0.0)), "max_rel": float(d.max(initial=0.0) / scale),
            "mean_abs": float(d.mean()) if d.size else 0.0, "cos": cos, "ref_absmax": scale,
            "finite": bool(np.isfinite(a).all())}


# ------------------------------------------------------------------------------------------------
# Seeded inputs for the five benchmark configurations (synthetic stand-ins for the reference's
# prot117/prot400 captures, which are not available here).
# ------------------------------------------------------------------------------------------------
CONFIGS = {
    0: dict(N=128, starting_only=True, dtype="fp32", z_scale=1.0, pad="none", seed_z=0, seed_w=0),
    1: dict(N=384, starting_only=False, dtype="fp16", z_scale=1.0, pad="fixed38", seed_z=1, seed_w=1),
    2: dict(N=1024, starting_only=False, dtype="bf16", z_scale=0.5, pad="uniform15", seed_z=2, seed_w=2),
    3: dict(N=768, starting_only=False, dtype="fp16", z_scale=1.0, pad="none", seed_z=3, seed_w=3, layers=128),
    4: dict(N=2048, starting_only=False, dtype="bf16", z_scale=1.0, pad="frac05", seed_z=4, seed_w=4),
}


def token_mask(N: int, pad: str, seed: int) -> torch.Tensor:
    """[N] token mask; the pair mask is its outer product (model.py:171-172)."""
    t = torch.ones(N)
    if pad == "fixed38":
        t[N - 38:] = 0
    elif pad == "uniform15":
        g = torch.Generator().manual_seed(10_000 + seed)
        n_pad = int(torch.randint(0, int(0.15 * N) + 1, (1,), generator=g))
        if n_pad:
            t[N - n_pad:] = 0
    elif pad == "frac05":
        t[N - int(round(0.05 * N)):] = 0
    return t


def make_inputs(cfg_id: int, *, N: Optional[int] = None, B: int = 1):
    """(z [B,N,N,128] fp32, pair mask [B,N,N] fp32, params) for a benchmark configuration."""
    c = CONFIGS[cfg_id]
    N = c["N"] if N is None else N
    g = torch.Generator().manual_seed(c["seed_z"])
    z = torch.randn((B, N, N, C_IN), generator=g) * c["z_scale"]
    t = token_mask(N, c["pad"], c["seed_z"])
    pm = (t[:, None] * t[None, :]).expand(B, N, N).contiguous()
    params = make_params(c["seed_w"], gate_bias=1.0)
    return z, pm, params
