"""TriangleAttention for B200: the reference's module interface over libtriattn.so.

Mirrors boltz_mlx/layers/triangular_attention/attention.py (jackryan225/boltz-mlx):
  * constructor  TriangleAttention(c_in, c_hidden, no_heads, starting=True, inf=1e9)   (attention.py:15)
  * parameters   layer_norm.{weight,bias}, linear.weight [H, c_in] (tri bias),
                 mha.linear_{q,k,v,g,o}.weight, no biases                              (attention.py:21-25,
                                                                                         primitives.py:33-38)
  * call         forward(x [B,I,J,c_in], mask [B,I,J] | None, chunk_size, use_kernels) -> update y
                 (the caller adds the residual, pairformer.py:86-87)                   (attention.py:27-35)
  * aliases      TriangleAttentionStartingNode / TriangleAttentionEndingNode           (attention.py:193-200)

Precision (the reference's BOLTZ_MLX_PRECISION = fp32 | f16, kernels.py:1216): `precision` is
"fp32" (SIMT fp32, the reference's fp32 path), "fp16" or "bf16" (tcgen05 tensor cores, fp32
accumulation).  Default: $TRIATTN_PRECISION or "fp32".

There is no CPU fallback: inputs must be CUDA tensors and libtriattn.so must be built.
"""

from __future__ import annotations

import os
from typing import Optional

import torch
from torch import nn

from . import _lib


class Attention(nn.Module):
    """Parameter container with the names of primitives.Attention (primitives.py:20-38)."""

    def __init__(self, c_q: int, c_k: int, c_v: int, c_hidden: int, no_heads: int, gating: bool = True):
        super().__init__()
        self.c_q, self.c_k, self.c_v, self.c_hidden, self.no_heads, self.gating = c_q, c_k, c_v, c_hidden, no_heads, gating
        self.linear_q = nn.Linear(c_q, c_hidden * no_heads, bias=False)
        self.linear_k = nn.Linear(c_k, c_hidden * no_heads, bias=False)
        self.linear_v = nn.Linear(c_v, c_hidden * no_heads, bias=False)
        self.linear_o = nn.Linear(c_hidden * no_heads, c_q, bias=False)
        if gating:
            self.linear_g = nn.Linear(c_q, c_hidden * no_heads, bias=False)


class Workspace:
    """Caller-owned device buffers of one layer call (the library never allocates)."""

    def __init__(self):
        self.buf: Optional[torch.Tensor] = None

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = None
            self.buf = torch.empty(nbytes, dtype=torch.uint8, device=device)
        return self.buf


def pack_weights(module: "TriangleAttention", dtype: int, stream: Optional[int] = None) -> torch.Tensor:
    """Pack a module's parameters into the library's layout (fp32 copies + tensor-core images)."""
    mha = module.mha
    dev = module.linear.weight.device
    f = lambda t: t.detach().to(device=dev, dtype=torch.float32).contiguous()
    ln_w = module.layer_norm.weight if module.layer_norm.weight is not None else torch.ones(module.c_in, device=dev)
    ln_b = module.layer_norm.bias if module.layer_norm.bias is not None else torch.zeros(module.c_in, device=dev)
    tensors = [f(ln_w), f(ln_b), f(mha.linear_q.weight), f(mha.linear_k.weight), f(mha.linear_v.weight),
               f(mha.linear_g.weight)]
    g_bias = f(mha.linear_g.bias) if getattr(mha.linear_g, "bias", None) is not None else None
    tensors += [g_bias, f(module.linear.weight), f(mha.linear_o.weight)]
    packed = torch.empty(_lib.packed_weights_bytes(dtype), dtype=torch.uint8, device=dev)
    st = _lib.stream_handle(dev) if stream is None else stream
    _lib.check(_lib.lib().triattn_pack_weights(*[_lib.ptr(t) for t in tensors], dtype, packed.data_ptr(),
                                              packed.numel(), st))
    module._pack_keepalive = tensors  # inputs stay alive until the (asynchronous) pack has run
    return packed


class TriangleAttention(nn.Module):
    """Triangle attention around the starting node (starting=True) or the ending node."""

    def __init__(self, c_in: int = 128, c_hidden: int = 32, no_heads: int = 4, starting: bool = True,
                 inf: float = 1e9, precision: Optional[str] = None) -> None:
        super().__init__()
        self.c_in, self.c_hidden, self.no_heads, self.starting, self.inf = c_in, c_hidden, no_heads, starting, inf
        self.layer_norm = nn.LayerNorm(c_in, eps=1e-5)
        self.linear = nn.Linear(c_in, no_heads, bias=False)
        self.mha = Attention(c_in, c_in, c_in, c_hidden, no_heads)
        self.precision = precision or os.environ.get("TRIATTN_PRECISION", "fp32")
        self._packed: dict = {}
        self._ws = Workspace()

    # ---- weights ----------------------------------------------------------------------------
    def _param_key(self):
        ps = [p for p in self.parameters()]
        return tuple((p.data_ptr(), p._version) for p in ps)

    def packed_weights(self, dtype: int) -> torch.Tensor:
        key = self._param_key()
        hit = self._packed.get(dtype)
        if hit is None or hit[0] != key:
            self._packed[dtype] = (key, pack_weights(self, dtype))
        return self._packed[dtype][1]

    def _check_geometry(self):
        if (self.c_in, self.c_hidden, self.no_heads) != (128, 32, 4) or not self.mha.gating:
            raise _lib.TriAttnUnsupported(
                _lib.EUNSUPPORTED,
                f"the sm_100a kernels implement c_in=128, 4 heads x 32 (got {self.c_in}, {self.no_heads}x{self.c_hidden})")

    # ---- calls ------------------------------------------------------------------------------
    def _run(self, x: torch.Tensor, mask: Optional[torch.Tensor], add_residual: bool,
             out: Optional[torch.Tensor]) -> torch.Tensor:
        self._check_geometry()
        if not x.is_cuda:
            raise RuntimeError("TriangleAttention (B200) needs CUDA tensors; there is no CPU path")
        if x.dim() != 4 or x.shape[1] != x.shape[2] or x.shape[3] != self.c_in:
            raise ValueError(f"x must be [B, N, N, {self.c_in}], got {tuple(x.shape)}")
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
        nbytes = _lib.workspace_bytes(B, N, N, dtype)
        ws = self._ws.get(nbytes, z.device)
        _lib.check(_lib.lib().triattn_forward(z.data_ptr(), _lib.ptr(m), packed.data_ptr(), B, N, int(self.starting),
                                              float(self.inf), dtype, int(add_residual), out.data_ptr(),
                                              ws.data_ptr(), ws.numel(), _lib.stream_handle(z.device)))
        return out

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None, chunk_size: Optional[int] = None,
                use_kernels: bool = False, xn: Optional[torch.Tensor] = None, keep_t: bool = False) -> torch.Tensor:
        """x [B, I, J, c_in] -> update y [B, I, J, c_in] (same orientation as x).

        `chunk_size` / `use_kernels` are accepted and ignored, as in the reference.  `xn` / `keep_t`
        belong to the reference's fused f16 pair block (attention.py:95-103); this build reads z in
        place in both orientations, so it takes neither."""
        if xn is not None or keep_t:
            raise _lib.TriAttnUnsupported(_lib.EUNSUPPORTED, "xn / keep_t (reference f16 pair-block plumbing)")
        return self._run(x, mask, False, None)

    def forward_residual(self, z: torch.Tensor, mask: Optional[torch.Tensor] = None, *,
                         inplace: bool = False) -> torch.Tensor:
        """z + self(z) in one pass (the pairformer's residual update, pairformer.py:86-87)."""
        zc = z.contiguous()
        out = zc if (inplace and zc is z and z.dtype == torch.float32) else None
        return self._run(zc, mask, True, out)


TriangleAttentionStartingNode = TriangleAttention


class TriangleAttentionEndingNode(TriangleAttention):
    """Triangle attention around the ending node (attention.py:196-200)."""

    def __init__(self, c_in: int = 128, c_hidden: int = 32, no_heads: int = 4, inf: float = 1e9,
                 precision: Optional[str] = None) -> None:
        super().__init__(c_in, c_hidden, no_heads, starting=False, inf=inf, precision=precision)


def load_params(module: TriangleAttention, params: dict) -> TriangleAttention:
    """Copy an oracle-style parameter dict (ln_w, ln_b, w_q, w_k, w_v, w_g, w_b, w_o, g_b) into the module."""
    with torch.no_grad():
        module.layer_norm.weight.copy_(params["ln_w"])
        module.layer_norm.bias.copy_(params["ln_b"])
        module.mha.linear_q.weight.copy_(params["w_q"])
        module.mha.linear_k.weight.copy_(params["w_k"])
        module.mha.linear_v.weight.copy_(params["w_v"])
        module.mha.linear_g.weight.copy_(params["w_g"])
        module.mha.linear_o.weight.copy_(params["w_o"])
        module.linear.weight.copy_(params["w_b"])
        if params.get("g_b") is not None:
            lg = module.mha.linear_g
            if lg.bias is None:
                lg.bias = nn.Parameter(torch.zeros(lg.out_features, device=lg.weight.device))
            lg.bias.copy_(params["g_b"])
    module._packed.clear()
    return module
