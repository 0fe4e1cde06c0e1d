"""GPU: triangle multiplication (outgoing / incoming) through libtriattn.so against the CPU oracle
(oracle/trimul_ref.py) on tiny / ragged N, B = 2, masked rows and columns; the fused residual (in
place) and the parameter names of the reference module.

Tolerances (max_rel = max|d| / max|ref|, the reference's compare metric):
  fp32  max_rel <= 1e-5 (the fp32 bar of the attention path)
  fp16  max_rel <= 3e-3, mean_abs <= 5e-3 (3e-3 is the reference's own bar between its two fp16
        tri-mult implementations, tests/test_nax2_kernels.py:162-173)
  bf16  max_rel <= 1e-2, mean_abs <= 5e-3 (bf16 keeps 3 mantissa bits fewer than fp16: x8 the rounding
        of xn, h, a, b and norm_out(o); the output of this layer reaches |y| ~ 3-4, so the attention
        path's absolute 2e-2 bar does not transfer)."""

import pytest
import torch

from boltz_mlx_b200 import TriangleMultiplicationIncoming, TriangleMultiplicationOutgoing, _lib, load_trimul_params
from oracle.triattn_ref import metrics
from oracle.trimul_ref import REF_NAMES, make_params, trimul_ref

MAX_REL = {"fp32": 1e-5, "fp16": 3e-3, "bf16": 1e-2}
MEAN_ABS = 5e-3


def assert_parity(out, ref, precision, name=""):
    m = metrics(out.detach().double().cpu().numpy(), ref.detach().double().cpu().numpy())
    assert m["finite"], f"{name}: non-finite output"
    assert m["max_rel"] <= MAX_REL[precision], f"{name}: {m}"
    if precision != "fp32":
        assert m["mean_abs"] <= MEAN_ABS, f"{name}: {m}"
    return m


pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status_clean():
    _lib.device_status(clear=True)
    yield
    assert _lib.device_status(clear=True) == 0


def _module(params, outgoing, precision):
    cls = TriangleMultiplicationOutgoing if outgoing else TriangleMultiplicationIncoming
    return load_trimul_params(cls(128, precision=precision).cuda(), params)


def _inputs(B, N, seed, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    z = scale * torch.randn(B, N, N, 128, generator=g)
    m = (torch.rand(B, N, N, generator=g) > 0.2).float()
    if N > 6:
        m[:, 3, :] = 0.0
        m[:, :, 5] = 0.0
    return z, m


@pytest.mark.parametrize("precision", ["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("B,N", [(1, 1), (1, 5), (2, 9), (1, 33), (1, 128), (1, 130)])
def test_trimul_vs_oracle(precision, outgoing, B, N):
    z, m = _inputs(B, N, 500 + N + B)
    p = make_params(11)
    ref = trimul_ref(z, m, p, outgoing=outgoing)
    out = _module(p, outgoing, precision)(z.cuda(), m.cuda())
    assert_parity(out, ref, precision, f"trimul out={outgoing} B={B} N={N}")


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_trimul_no_mask_and_residual_in_place(precision):
    z, _ = _inputs(1, 40, 7)
    p = make_params(12)
    for outgoing in (True, False):
        mod = _module(p, outgoing, precision)
        zc = z.cuda()
        y = mod(zc, None)
        assert torch.equal(y, mod(zc, torch.ones(1, 40, 40, device="cuda")))
        assert_parity(y, trimul_ref(z, None, p, outgoing=outgoing), precision, "no mask")
        zi = zc.clone()
        r = mod.forward_residual(zi, None, inplace=True)
        assert r.data_ptr() == zi.data_ptr()
        assert torch.allclose(zi, zc + y, rtol=0, atol=1e-5 if precision == "fp32" else 1e-5)


def test_trimul_bench_size_bf16():
    """The pair size of the benchmark's smaller config (N = 384, bf16), both directions."""
    z, m = _inputs(1, 384, 3, scale=0.5)
    m[:, :, 350:] = 0.0
    m[:, 350:, :] = 0.0
    p = make_params(13)
    for outgoing in (True, False):
        out = _module(p, outgoing, "bf16")(z.cuda(), m.cuda())
        assert_parity(out, trimul_ref(z, m, p, outgoing=outgoing), "bf16", f"N=384 out={outgoing}")


def test_trimul_parameter_names_match_reference():
    mod = TriangleMultiplicationOutgoing(128)
    assert sorted(n for n, _ in mod.named_parameters()) == sorted(REF_NAMES.values())


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
def test_trimul_f16_addln_feeds_the_next_layernorm(precision):
    """f16_addln: z + y equals forward_residual bit for bit, and ln_out equals the next module's
    LayerNorm of it (fp32 statistics, one 16-bit rounding); the next tri bias from w_tb."""
    z, m = _inputs(1, 70, 17)
    p = make_params(14)
    ln = torch.nn.LayerNorm(128, eps=1e-5).cuda()
    with torch.no_grad():
        ln.weight.copy_(1.0 + 0.1 * torch.randn(128))
        ln.bias.copy_(0.1 * torch.randn(128))
    w_tb = torch.randn(4, 128).cuda() / 128 ** 0.5
    t16 = torch.bfloat16 if precision == "bf16" else torch.float16
    for outgoing in (True, False):
        mod = _module(p, outgoing, precision)
        zc, mc = z.cuda(), m.cuda()
        z_new, ln_out, tb = mod.f16_addln(zc, mc, None, ln, w_tb=w_tb)
        assert torch.equal(z_new, mod.forward_residual(zc, mc))
        ref = torch.nn.functional.layer_norm(z_new, (128,), ln.weight, ln.bias, 1e-5)
        assert ln_out.dtype == t16
        d = (ln_out.float() - ref).abs()
        tol = 1e-2 if precision == "bf16" else 2e-3
        assert float(d.max()) <= tol * max(1.0, float(ref.abs().max())), float(d.max())
        # the next tri bias from the tail kernel: fp32 sums of the rounded ln_out, one rounding to fp16
        assert tb.shape == (1, 4, 70, 70) and tb.dtype == torch.float16
        tb_ref = (ln_out.float() @ w_tb.t()).permute(0, 3, 1, 2)
        assert ((tb.float() - tb_ref).abs() <= 2.0 ** -11 * tb_ref.abs() + 1e-5).all()
    with pytest.raises(_lib.TriAttnUnsupported):
        _module(p, True, "fp32").f16_addln(z.cuda(), m.cuda(), None, ln)
