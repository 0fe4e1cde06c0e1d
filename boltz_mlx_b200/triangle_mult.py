"""TriangleMultiplication{Outgoing,Incoming} for B200: the reference's module interface over
libtriattn.so (triattn_trimul_*).

Mirrors boltz_mlx/layers/triangular_mult.py (jackryan225/boltz-mlx):
  * constructor  TriangleMultiplicationOutgoing(dim=128) / TriangleMultiplicationIncoming(dim=128)
                                                                             (triangular_mult.py:13-21, 173-178)
  * parameters   norm_in.{weight,bias}, p_in.weight [256,128], g_in.weight [256,128],
                 norm_out.{weight,bias}, p_out.weight [128,128], g_out.weight [128,128], no biases
  * call         forward(x [B,N,N,128], mask [B,N,N], use_kernels=False, xn=None) -> update y
                 (the pairformer adds the residual)                          (triangular_mult.py:23-49)

`precision` "fp32" runs every step in fp32; "fp16" / "bf16" keep the projections and the contraction
operands 16-bit with fp32 accumulation and an fp32 contraction output.  There is no CPU fallback.
"""

from __future__ import annotations

import os
from typing import Optional

import torch
from torch import nn

from . import _lib
from .triangle_attention import Workspace


class _TriangleMultiplication(nn.Module):
    outgoing: bool = True

    def __init__(self, dim: int = 128, precision: Optional[str] = None) -> None:
        super().__init__()
        self.dim = dim
        self.norm_in = nn.LayerNorm(dim, eps=1e-5)
        self.p_in = nn.Linear(dim, 2 * dim, bias=False)
        self.g_in = nn.Linear(dim, 2 * dim, bias=False)
        self.norm_out = nn.LayerNorm(dim, eps=1e-5)
        self.p_out = nn.Linear(dim, dim, bias=False)
        self.g_out = nn.Linear(dim, dim, bias=False)
        self.precision = precision or os.environ.get("TRIATTN_PRECISION", "fp32")
        self._packed: dict = {}
        self._ws = Workspace()

    def _param_key(self):
        return tuple((p.data_ptr(), p._version) for p in self.parameters())

    def packed_weights(self, dtype: int) -> torch.Tensor:
        key = self._param_key()
        hit = self._packed.get(dtype)
        if hit is None or hit[0] != key:
            dev = self.p_in.weight.device
            f = lambda t: t.detach().to(device=dev, dtype=torch.float32).contiguous()
            ts = [f(self.norm_in.weight), f(self.norm_in.bias), f(self.p_in.weight), f(self.g_in.weight),
                  f(self.norm_out.weight), f(self.norm_out.bias), f(self.p_out.weight), f(self.g_out.weight)]
            packed = torch.empty(_lib.lib().triattn_trimul_packed_bytes(dtype), dtype=torch.uint8, device=dev)
            _lib.check(_lib.lib().triattn_trimul_pack_weights(*[t.data_ptr() for t in ts], dtype, packed.data_ptr(),
                                                             packed.numel(), _lib.stream_handle(dev)))
            self._pack_keepalive = ts  # inputs stay alive until the (asynchronous) pack has run
            self._packed[dtype] = (key, packed)
        return self._packed[dtype][1]

    def _run(self, x: torch.Tensor, mask: Optional[torch.Tensor], add_residual: bool,
             out: Optional[torch.Tensor]) -> torch.Tensor:
        if self.dim != 128:
            raise _lib.TriAttnUnsupported(_lib.EUNSUPPORTED, f"the sm_100a kernels implement dim=128 (got {self.dim})")
        if not x.is_cuda:
            raise RuntimeError("TriangleMultiplication (B200) needs CUDA tensors; there is no CPU path")
        if x.dim() != 4 or x.shape[1] != x.shape[2] or x.shape[3] != self.dim:
            raise ValueError(f"x must be [B, N, N, {self.dim}], got {tuple(x.shape)}")
        dtype = _lib.dtype_code(self.precision)
        z = x.contiguous() if x.dtype == torch.float32 else x.float().contiguous()
        B, N = z.shape[0], z.shape[1]
        m = None
        if mask is not None:
            if tuple(mask.shape) != (B, N, N):
                raise ValueError(f"mask must be [B, N, N] = {(B, N, N)}, got {tuple(mask.shape)}")
            m = mask.to(device=z.device, dtype=torch.float32).contiguous()
        if out is None:
            out = torch.empty_like(z)
        packed = self.packed_weights(dtype)
        ws = self._ws.get(_lib.lib().triattn_trimul_workspace_bytes(B, N, dtype), z.device)
        _lib.check(_lib.lib().triattn_trimul_forward(z.data_ptr(), _lib.ptr(m), packed.data_ptr(), B, N,
                                                     int(self.outgoing), dtype, int(add_residual), out.data_ptr(),
                                                     ws.data_ptr(), ws.numel(), _lib.stream_handle(z.device)))
        return out

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None, use_kernels: bool = False,
                xn: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x [B, N, N, 128] -> update y [B, N, N, 128] (triangular_mult.py:23-49).  `use_kernels` is accepted
        and ignored, as in the reference; `xn` (a precomputed norm_in(x)) is accepted and recomputed here
        from x, which the output gate's projection needs anyway."""
        del use_kernels, xn
        return self._run(x, mask, False, None)

    def forward_residual(self, z: torch.Tensor, mask: Optional[torch.Tensor] = None, *,
                         inplace: bool = False) -> torch.Tensor:
        """z + self(z) in one pass (the pairformer's residual update)."""
        zc = z.contiguous()
        out = zc if (inplace and zc is z and z.dtype == torch.float32) else None
        return self._run(zc, mask, True, out)

    def f16_addln(self, z: torch.Tensor, mask: Optional[torch.Tensor], xn: Optional[torch.Tensor], ln_next,
                  w_tb: Optional[torch.Tensor] = None):
        """(z + self(z), ln_next(z + self(z)) 16-bit[, next tri bias]) as the reference's f16_addln
        (triangular_mult.py:93-115): the output gate, the residual add and the next module's LayerNorm in
        the tail kernel.  16-bit precisions only.  `xn` (norm_in(z), precomputed) is accepted and
        recomputed from z.  `w_tb` [H, 128] (the next triangle attention's tb_weight16()): also return
        that module's tri bias, computed in the tail kernel's epilogue from the rounded 16-bit LayerNorm
        rows (fp32 sums, one rounding to fp16), as [B, H, N, N] (the reference's PAIRTB,
        kernels_nax3.py:104-143)."""
        del xn
        if not z.is_cuda:
            raise RuntimeError("TriangleMultiplication (B200) needs CUDA tensors; there is no CPU path")
        dtype = _lib.dtype_code(self.precision)
        if dtype == _lib.F32:
            raise _lib.TriAttnUnsupported(_lib.EUNSUPPORTED, "f16_addln belongs to the 16-bit path (fp16 or bf16)")
        if z.dim() != 4 or z.shape[1] != z.shape[2] or z.shape[3] != self.dim or z.dtype != torch.float32:
            raise ValueError(f"z must be fp32 [B, N, N, {self.dim}], got {tuple(z.shape)} {z.dtype}")
        zc = z.contiguous()
        B, N = zc.shape[0], zc.shape[1]
        m = None
        if mask is not None:
            if tuple(mask.shape) != (B, N, N):
                raise ValueError(f"mask must be [B, N, N] = {(B, N, N)}, got {tuple(mask.shape)}")
            m = mask.to(device=zc.device, dtype=torch.float32).contiguous()
        t16 = torch.bfloat16 if dtype == _lib.BF16 else torch.float16
        lw = ln_next.weight.detach().to(device=zc.device, dtype=torch.float32).contiguous()
        lb = ln_next.bias.detach().to(device=zc.device, dtype=torch.float32).contiguous()
        out = torch.empty_like(zc)
        ln_out = torch.empty(zc.shape, dtype=t16, device=zc.device)
        wt, tb_next = None, None
        if w_tb is not None:
            if w_tb.dim() != 2 or w_tb.shape[1] != self.dim:
                raise ValueError(f"w_tb must be [H, {self.dim}], got {tuple(w_tb.shape)}")
            if w_tb.shape[0] != 4:
                raise _lib.TriAttnUnsupported(_lib.EUNSUPPORTED, "the tail kernel writes the tri bias of 4 heads")
            wt = w_tb.detach().to(device=zc.device, dtype=torch.float32).contiguous()
            tb_next = torch.empty(B, 4, N, N, dtype=torch.float16, device=zc.device)
        packed = self.packed_weights(dtype)
        ws = self._ws.get(_lib.lib().triattn_trimul_workspace_bytes(B, N, dtype), zc.device)
        _lib.check(_lib.lib().triattn_trimul_forward_addln_tb(
            zc.data_ptr(), _lib.ptr(m), packed.data_ptr(), B, N, int(self.outgoing), dtype, out.data_ptr(),
            lw.data_ptr(), lb.data_ptr(), ln_out.data_ptr(), _lib.ptr(wt), _lib.ptr(tb_next), ws.data_ptr(), ws.numel(),
            _lib.stream_handle(zc.device)))
        if w_tb is None:
            return out, ln_out
        return out, ln_out, tb_next


class TriangleMultiplicationOutgoing(_TriangleMultiplication):
    """o[i,j] = sum_k a[i,k] b[j,k] (triangular_mult.py:173-174)."""

    outgoing = True


class TriangleMultiplicationIncoming(_TriangleMultiplication):
    """o[i,j] = sum_k a[k,i] b[k,j] (triangular_mult.py:177-178)."""

    outgoing = False


def load_trimul_params(module: _TriangleMultiplication, params: dict) -> _TriangleMultiplication:
    """Copy an oracle-style parameter dict (in_w, in_b, p_in, g_in, out_w, out_b, p_out, g_out) into the
    module's reference-named parameters."""
    names = {"in_w": module.norm_in.weight, "in_b": module.norm_in.bias, "p_in": module.p_in.weight,
             "g_in": module.g_in.weight, "out_w": module.norm_out.weight, "out_b": module.norm_out.bias,
             "p_out": module.p_out.weight, "g_out": module.g_out.weight}
    with torch.no_grad():
        for k, p in names.items():
            p.copy_(params[k].to(device=p.device, dtype=p.dtype))
    return module
