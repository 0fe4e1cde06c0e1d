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

import contextlib
import warnings

from . import _lib
from .layout import workspace_bytes


@contextlib.contextmanager
def nvtx_range(name: str):
    """An NVTX range around one layer call (visible in Nsight timelines); a no-op where NVTX is absent."""
    pushed = False
    try:
        torch.cuda.nvtx.range_push(name)
        pushed = True
    except Exception:  # noqa: BLE001 - tracing must never break a call
        pass
    try:
        yield
    finally:
        if pushed:
            try:
                torch.cuda.nvtx.range_pop()
            except Exception:  # noqa: BLE001
                pass


def run_with_fp32_fallback(run16, run32, all_finite) -> tuple:
    """The reference's overflow guard (model.py:179-193: a 16-bit overflow triggers a recompute in
    fp32), as control flow: run the 16-bit layer; if its output is not all finite, run the fp32 layer.
    Returns (output, fell_back)."""
    out = run16()
    if all_finite(out):
        return out, False
    return run32(), True


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

    # Workspace budget of one call: a layer whose full workspace is larger runs row-chunked (the tri
    # bias of all rows, then chunks of rows; attention.py:55-68).  At B = 1, 16-bit: N = 2048 needs
    # 5.4 GB and runs whole; N = 4096 needs 21 GB and runs in chunks.
    max_workspace_bytes: int = 8 << 30
    # 16-bit precisions: check each output for inf / nan (one reduction and a host sync per call) and
    # recompute the layer in fp32 when any is found, as the reference does on an fp16 overflow
    fp32_fallback: bool = False
    nonfinite_events: int = 0

    def chunk_rows(self, B: int, N: int, dtype: int, chunk_size: Optional[int] = None) -> int:
        """Rows per chunk for a B x N layer: `chunk_size` rounded up to a whole 128-row tile on the
        16-bit path, or (None) all N rows when the workspace fits max_workspace_bytes, else the
        largest multiple of 128 rows that fits (at least 128)."""
        if chunk_size is not None:
            if chunk_size < 1:
                raise ValueError(f"chunk_size must be >= 1, got {chunk_size}")
            c = chunk_size if dtype == _lib.F32 else -(-chunk_size // 128) * 128
            return min(c, N)
        if workspace_bytes(B, N, N, dtype) <= self.max_workspace_bytes:
            return N
        c = 128
        while c + 128 < N and workspace_bytes(B, N, c + 128, dtype) <= self.max_workspace_bytes:
            c += 128
        return min(c, N)

    # ---- calls ------------------------------------------------------------------------------
    def _run(self, x: torch.Tensor, mask: Optional[torch.Tensor], add_residual: bool,
             out: Optional[torch.Tensor], chunk_size: Optional[int] = None) -> torch.Tensor:
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

        def launch(dt: int, dst: torch.Tensor) -> torch.Tensor:
            packed = self.packed_weights(dt)
            rows = self.chunk_rows(B, N, dt, chunk_size)
            ws = self._ws.get(_lib.workspace_bytes(B, N, rows, dt), z.device)
            if rows == N:
                _lib.check(_lib.lib().triattn_forward(z.data_ptr(), _lib.ptr(m), packed.data_ptr(), B, N,
                                                      int(self.starting), float(self.inf), dt, int(add_residual),
                                                      dst.data_ptr(), ws.data_ptr(), ws.numel(),
                                                      _lib.stream_handle(z.device)))
            else:
                _lib.check(_lib.lib().triattn_forward_chunked(z.data_ptr(), _lib.ptr(m), packed.data_ptr(), B, N,
                                                              int(self.starting), float(self.inf), dt,
                                                              int(add_residual), dst.data_ptr(), rows,
                                                              ws.data_ptr(), ws.numel(), _lib.stream_handle(z.device)))
            return dst

        with nvtx_range(f"triattn.{'start' if self.starting else 'end'}"):
            if not self.fp32_fallback or dtype == _lib.F32:
                return launch(dtype, out)
            # guarded: never overwrite z in place before the 16-bit result is known to be finite
            dst = torch.empty_like(z) if out.data_ptr() == z.data_ptr() else out
            res, fell_back = run_with_fp32_fallback(lambda: launch(dtype, dst), lambda: launch(_lib.F32, dst),
                                                    lambda t: bool(torch.isfinite(t).all()))
            if fell_back:
                self.nonfinite_events += 1
                warnings.warn(f"TriangleAttention: non-finite {self.precision} output at N={N}; recomputed in fp32",
                              RuntimeWarning, stacklevel=3)
            if dst is not out:
                out.copy_(res)
            return out

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None, chunk_size: Optional[int] = None,
                use_kernels: bool = False, xn: Optional[torch.Tensor] = None, keep_t: bool = False) -> torch.Tensor:
        """x [B, I, J, c_in] -> update y [B, I, J, c_in] (same orientation as x).

        `chunk_size`: rows per chunk of the row-chunked layer (None: automatic, whole layer unless its
        workspace exceeds max_workspace_bytes); the result is the same bit for bit either way.
        `use_kernels` is accepted and ignored, as in the reference.  As in the reference's
        f16 path (attention.py:95-103): `xn` = this module's LayerNorm output already computed (16-bit, the
        module's type; for the ending node already transposed), so the LayerNorm is skipped; `keep_t` =
        return the ending node's update in the transposed layout."""
        if xn is None and not keep_t:
            return self._run(x, mask, False, None, chunk_size)
        return self._run_fused(x, mask, xn, add_residual=False, keep_t=keep_t)[0]

    def f16_addln(self, z: torch.Tensor, mask: Optional[torch.Tensor], xn: Optional[torch.Tensor], ln_next,
                  trans_out: bool = False, tb: Optional[torch.Tensor] = None, w_tb: Optional[torch.Tensor] = None):
        """(z + self(z), ln_next(z + self(z)) 16-bit [transposed with trans_out][, next tri bias]) as the
        reference's f16_addln (attention.py:170-190, kernels_nax3.linear_addln): the layer from
        xn = this module's LayerNorm output (ending node: already transposed), then the output projection,
        the residual add and the next module's LayerNorm in the output kernel's epilogue.

        `ln_next`: a LayerNorm module (weight, bias; eps 1e-5).  `tb` [B, H, N, N]: this module's tri bias
        computed by the producer of xn (laid out like xn; fp16 in natural units), used by the projection
        instead of its own LN . w_b dot (attention.py:128-147).  `w_tb` [H, c_in] (the next triangle
        attention's tb_weight16()): also return that module's tri bias, computed in the output kernel's
        epilogue from the rounded 16-bit LayerNorm rows (fp32 sums, one rounding to fp16), as
        [B, H, Q, K] in ln_out's layout (the reference's PAIRTB, kernels_nax3.py:104-143)."""
        z_new, ln_out, tb_next = self._run_fused(z, mask, xn, add_residual=True, keep_t=False, ln_next=ln_next,
                                                 trans_out=trans_out, tb=tb, w_tb=w_tb)
        if w_tb is None:
            return z_new, ln_out
        return z_new, ln_out, tb_next

    def tb_weight16(self) -> torch.Tensor:
        """The tri-bias projection weight [H, c_in] rounded to fp16, as the reference passes it to the
        producer's f16_addln(w_tb=...) (attention.py:158-164)."""
        return self.linear.weight.detach().to(torch.float16)

    def _run_fused(self, x, mask, xn, *, add_residual: bool, keep_t: bool, ln_next=None, trans_out: bool = False,
                   tb=None, w_tb=None):
        self._check_geometry()
        if not x.is_cuda:
            raise RuntimeError("TriangleAttention (B200) needs CUDA tensors; there is no CPU path")
        dtype = _lib.dtype_code(self.precision)
        if dtype == _lib.F32:
            raise _lib.TriAttnUnsupported(_lib.EUNSUPPORTED,
                                          "xn / keep_t / f16_addln belong to the 16-bit path (precision fp16 or bf16)")
        t16 = torch.bfloat16 if dtype == _lib.BF16 else torch.float16
        z = x.contiguous() if x.dtype == torch.float32 else x.float().contiguous()
        B, N = z.shape[0], z.shape[1]
        if z.dim() != 4 or z.shape[2] != N or z.shape[3] != self.c_in:
            raise ValueError(f"x must be [B, N, N, {self.c_in}], got {tuple(z.shape)}")
        if xn is not None:
            if tuple(xn.shape) != tuple(z.shape):
                raise ValueError(f"xn must be {tuple(z.shape)}, got {tuple(xn.shape)}")
            xn = xn.to(device=z.device, dtype=t16).contiguous()
        m = None
        if mask is not None:
            if tuple(mask.shape) != (B, N, N):
                raise ValueError(f"mask must be [B, N, N] = {(B, N, N)}, got {tuple(mask.shape)}")
            m = mask.to(device=z.device, dtype=torch.float32).contiguous()
        out = torch.empty_like(z)
        ln_out, lw, lb = None, None, None
        if ln_next is not None:
            lw = ln_next.weight.detach().to(device=z.device, dtype=torch.float32).contiguous()
            lb = ln_next.bias.detach().to(device=z.device, dtype=torch.float32).contiguous()
            ln_out = torch.empty(z.shape, dtype=t16, device=z.device)
        H = self.no_heads
        if tb is not None:
            if xn is None:
                raise ValueError("tb (the producer's tri bias) comes with xn, the producer's LayerNorm output")
            if tuple(tb.shape) != (B, H, N, N):
                raise ValueError(f"tb must be [B, H, N, N] = {(B, H, N, N)}, got {tuple(tb.shape)}")
            tb = tb.to(device=z.device, dtype=torch.float16).contiguous()
        wt, tb_next = None, None
        if w_tb is not None:
            if ln_next is None:
                raise ValueError("w_tb needs ln_next: the next tri bias is computed from the next LayerNorm's output")
            if tuple(w_tb.shape) != (H, self.c_in):
                raise ValueError(f"w_tb must be [H, c_in] = {(H, self.c_in)}, got {tuple(w_tb.shape)}")
            wt = w_tb.detach().to(device=z.device, dtype=torch.float32).contiguous()
            tb_next = torch.empty(B, H, N, N, dtype=torch.float16, device=z.device)
        packed = self.packed_weights(dtype)
        nbytes = _lib.workspace_bytes(B, N, N, dtype)
        ws = self._ws.get(nbytes, z.device)
        out_attn = int(keep_t and not self.starting)
        _lib.check(_lib.lib().triattn_forward_fused_tb(
            z.data_ptr(), _lib.ptr(xn), _lib.ptr(tb), _lib.ptr(m), packed.data_ptr(), B, N, int(self.starting),
            float(self.inf), dtype, int(add_residual), out.data_ptr(), out_attn, _lib.ptr(lw), _lib.ptr(lb),
            _lib.ptr(ln_out), int(trans_out), _lib.ptr(wt), _lib.ptr(tb_next), ws.data_ptr(), ws.numel(),
            _lib.stream_handle(z.device)))
        self._fused_keepalive = (xn, tb, m, lw, lb, wt)  # inputs stay alive until the (asynchronous) launch has run
        return out, ln_out, tb_next

    def forward_residual(self, z: torch.Tensor, mask: Optional[torch.Tensor] = None, *,
                         inplace: bool = False, chunk_size: Optional[int] = None) -> torch.Tensor:
        """z + self(z) in one pass (the pairformer's residual update, pairformer.py:86-87)."""
        zc = z.contiguous()
        out = zc if (inplace and zc is z and z.dtype == torch.float32) else None
        return self._run(zc, mask, True, out, chunk_size)


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
