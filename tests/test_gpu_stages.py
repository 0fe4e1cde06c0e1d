"""GPU: each stage of the 16-bit tensor-core path, through the C ABI, against a torch fp32 computation
of the same stage on the same inputs (16-bit rounding points reproduced).  A layout or descriptor
mistake shows up here in the stage that makes it."""

import pytest
import torch

from boltz_mlx_b200 import _lib, layout
from oracle.triattn_ref import C_HEAD, HC, HEADS, LN_EPS, make_params
from tests._util import module, rand_mask

pytestmark = pytest.mark.gpu
LOG2E = 1.4426950408889634
QSCALE_L2 = C_HEAD ** -0.5 * LOG2E  # q is stored pre-scaled: S = q.k comes out in log2 units


def t16(precision):
    return torch.bfloat16 if precision == "bf16" else torch.float16


def run_ln_proj(N, precision, starting=True, B=1, seed=0, mask=None):
    dt = _lib.dtype_code(precision)
    g = torch.Generator().manual_seed(seed + N)
    z = torch.randn(B, N, N, 128, generator=g)
    p = make_params(seed + N, gate_bias=1.0, ln_identity=False)
    mod = module(p, starting, precision)
    packed = mod.packed_weights(dt)
    w = layout.Workspace.make(B, N, N, dt)
    ws = torch.full((w.total,), 0xFF, dtype=torch.uint8, device="cuda")  # poison: unwritten bytes are NaN
    zc = z.cuda()
    mc = None if mask is None else mask.cuda()
    L = _lib.lib()
    st = _lib.stream_handle(zc.device)
    _lib.check(L.triattn_mask_prep(_lib.ptr(mc), B, N, int(starting), 1e9, 0, N, dt, ws.data_ptr(), ws.numel(), st))
    _lib.check(L.triattn_ln_proj(zc.data_ptr(), packed.data_ptr(), B, N, int(starting), 0, N, dt, ws.data_ptr(),
                                 ws.numel(), st))
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    return dict(z=z, p=p, mod=mod, packed=packed, w=w, ws=ws, zc=zc, dt=dt, mask=mask, B=B, N=N, starting=starting)


def ref_projection(ctx, precision):
    z, p = ctx["z"], ctx["p"]
    x = z if ctx["starting"] else z.transpose(1, 2)
    mu = x.mean(-1, keepdim=True)
    var = ((x - mu) ** 2).mean(-1, keepdim=True)
    xn = (x - mu) / torch.sqrt(var + LN_EPS) * p["ln_w"] + p["ln_b"]
    r = lambda t: t.to(t16(precision)).float()
    W = torch.cat([p["w_q"], p["w_k"], p["w_v"], p["w_g"]], 0)
    h = r(xn) @ r(W).T  # 16-bit operands, fp32 accumulate
    tb = xn @ p["w_b"].T  # fp32 SIMT dot in the kernel
    return xn, h, tb


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
@pytest.mark.parametrize("N,starting", [(9, True), (128, True), (200, False), (129, True)])
def test_ln_proj_stage(precision, N, starting):
    ctx = run_ln_proj(N, precision, starting)
    w, ws, B = ctx["w"], ctx["ws"], ctx["B"]
    xn, h, tb = ref_projection(ctx, precision)
    # a 16-bit ulp: accumulation order and 1-ulp LN differences flip the last rounding of a few values
    ulp = 2.0 ** -8 if precision == "bf16" else 2.0 ** -11
    f16ulp = 2.0 ** -11
    for i, off in enumerate((w.off_q, w.off_k)):
        img = layout.decode_head_images(ws, w, off).cpu()  # [B, R, H, Np, 32]
        ref = h[..., i * HC:(i + 1) * HC].reshape(B, N, N, HEADS, C_HEAD).permute(0, 1, 3, 2, 4)
        if i == 0:
            ref = ref * QSCALE_L2
        got = img[:, :, :, :N]
        torch.testing.assert_close(got, ref.to(t16(precision)).float(), rtol=2 * ulp,
                                   atol=ulp * float(ref.abs().max()), msg=lambda m: f"image {i}: {m}")
        assert torch.all(img[:, :, :, N:] == 0), "padded positions must be zero"
    vimg = layout.decode_v_images(ws, w).cpu()
    vref = h[..., 2 * HC:3 * HC].reshape(B, N, N, HEADS, C_HEAD).permute(0, 1, 3, 2, 4)
    # V is fp16 in every 16-bit mode; its operand is the bf16/fp16-rounded xn, so compare at that ulp
    torch.testing.assert_close(vimg[:, :, :, :N], vref.half().float(), rtol=2 * max(ulp, f16ulp),
                               atol=ulp * float(vref.abs().max()))
    assert torch.all(vimg[:, :, :, N:] == 0)
    gbuf = ws[w.off_g:w.off_g + B * N * N * 128 * 2].view(t16(precision)).view(B, N, N, 128).float().cpu()
    gref = (h[..., 3 * HC:] + 1.0).to(t16(precision)).float()
    torch.testing.assert_close(gbuf, gref, rtol=2 * ulp, atol=ulp * float(gref.abs().max()))
    bias = layout.decode_bias16(ws, w).cpu()  # [B, H, q, k]
    ref_b = (tb * LOG2E).permute(0, 3, 1, 2)  # tb [B, q, k, H]
    torch.testing.assert_close(bias, ref_b.half().float(), rtol=2 * f16ulp, atol=1e-4)


def ref_core(ctx, precision):
    """Softmax attention on the decoded operand images, fp32, log2 domain (kernels_nax.py:376-406):
    S = q'.k (q' pre-scaled), x = S + mask bias + tri bias, p = 2^(x - max), o = p v / sum p (the core
    stage stores o; the sigmoid gate is applied by the output projection)."""
    w, ws, B, N = ctx["w"], ctx["ws"], ctx["B"], ctx["N"]
    q = layout.decode_head_images(ws, w, w.off_q)[:, :, :, :N].cpu()
    k = layout.decode_head_images(ws, w, w.off_k)[:, :, :, :N].cpu()
    v = layout.decode_v_images(ws, w)[:, :, :, :N].cpu()
    bias = layout.decode_bias16(ws, w).cpu()  # [B, H, q, k]
    mb = ws[w.off_mb:w.off_mb + B * N * w.Np * 4].view(torch.float32).view(B, N, w.Np).cpu()
    s = torch.einsum("bahqd,bahkd->bahqk", q, k)
    s = (s + mb[:, :, None, None, :N]) + bias[:, None]
    s = s - s.amax(-1, keepdim=True)
    pr = torch.exp2(s)
    o = torch.einsum("bahqk,bahkd->bahqd", pr, v) / pr.sum(-1, keepdim=True)
    return o.permute(0, 1, 3, 2, 4).reshape(B, N, N, HC)


def test_tile_classes():
    """Key-tile classes: 0 all valid, 1 all masked with valid keys elsewhere (skipped), 2 mixed or a
    row without any valid key (kept, so it attends uniformly)."""
    N = 300
    mask = torch.ones(1, N, N)
    mask[0, 0, 128:256] = 0  # row 0: tile 1 fully masked -> skipped
    mask[0, 1, 5] = 0  # row 1: tile 0 mixed
    mask[0, 2, :] = 0  # row 2: no valid key -> every tile kept
    ctx = run_ln_proj(N, "bf16", True, mask=mask)
    w, ws = ctx["w"], ctx["ws"]
    ts = ws[w.off_ts:w.off_ts + N * w.NTs].view(N, w.NTs)[:, :w.NT].cpu().tolist()
    assert w.NT == 3
    assert ts[0] == [0, 1, 2]  # the last tile holds padded keys -> mixed
    assert ts[1] == [2, 0, 2]
    assert ts[2] == [2, 2, 2]
    assert ts[3] == [0, 0, 2]


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
@pytest.mark.parametrize("N,masked", [(9, False), (128, True), (200, True), (300, False)])
def test_core_stage(precision, N, masked):
    g = torch.Generator().manual_seed(77 + N)
    mask = rand_mask(g, 1, N, "rows_cols") if masked else None
    ctx = run_ln_proj(N, precision, True, mask=mask)
    w, ws = ctx["w"], ctx["ws"]
    _lib.check(_lib.lib().triattn_core(1, N, 0, N, ctx["dt"], ws.data_ptr(), ws.numel(),
                                       _lib.stream_handle(ws.device)))
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    got = layout.decode_core_images(ws, w)[:, :, :N].cpu()
    ref = ref_core(ctx, precision)
    assert torch.isfinite(got).all()
    err = (got - ref).abs()
    scale = ref.abs().max()
    assert err.max() <= 2e-2 * scale and err.mean() <= 2e-3 * scale, (float(err.max()), float(err.mean()), float(scale))


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
@pytest.mark.parametrize("starting,residual", [(True, False), (False, True)])
def test_out_proj_stage(precision, starting, residual):
    N = 140
    ctx = run_ln_proj(N, precision, starting)
    w, ws, L = ctx["w"], ctx["ws"], _lib.lib()
    st = _lib.stream_handle(ws.device)
    _lib.check(L.triattn_core(1, N, 0, N, ctx["dt"], ws.data_ptr(), ws.numel(), st))
    out = torch.full_like(ctx["zc"], float("nan"))
    _lib.check(L.triattn_out_proj(ctx["zc"].data_ptr(), ctx["packed"].data_ptr(), 1, N, int(starting), 0, N, ctx["dt"],
                                  int(residual), out.data_ptr(), ws.data_ptr(), ws.numel(), st))
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    core = layout.decode_core_images(ws, w)[:, :, :N].cpu()
    g = ws[w.off_g:w.off_g + N * N * 128 * 2].view(t16(precision)).view(1, N, N, 128).float().cpu()
    gated = core * torch.sigmoid(g)  # rounded once to the 16-bit type inside the kernel
    wo = ctx["p"]["w_o"].to(t16(precision)).float()
    y = gated @ wo.T  # attention orientation
    # one rounding of each gated value (half an ulp, relative) bounds the difference
    rel = 2.0 ** -8 if precision == "bf16" else 2.0 ** -11
    bound = 1.5 * rel * (gated.abs() @ wo.abs().T) + 1e-5
    if not starting:
        y, bound = y.transpose(1, 2), bound.transpose(1, 2)
    if residual:
        y = y + ctx["z"]
        bound = bound + 1e-6 * ctx["z"].abs()
    err = (out.cpu() - y).abs()
    assert torch.isfinite(out.cpu()).all()
    assert (err <= bound).all(), float((err - bound).max())
