"""GPU: the reference's fused f16 pair-block plumbing (attention.py:95-103,170-190; kernels_nax3.py:69-198;
kernels.py:1526-1547) through triattn_forward_fused: a caller-given LayerNorm output `xn` (LayerNorm
skipped), `keep_t` (ending-node update in the transposed layout) and `f16_addln` (residual add and the
next module's LayerNorm in the output kernel), checked against the float64 oracle and against the
plain path."""

import pytest
import torch
import torch.nn.functional as F

from oracle.triattn_ref import make_params, tri_attention_ref
from tests._util import assert_parity, module, rand_mask

pytestmark = pytest.mark.gpu
T16 = {"bf16": torch.bfloat16, "fp16": torch.float16}


def _ln16(z, ln, starting, precision):
    """The module's LayerNorm output in its attention orientation (ending node: transposed), 16-bit."""
    x = z if starting else z.transpose(1, 2)
    return F.layer_norm(x, (128,), ln.weight, ln.bias, 1e-5).to(T16[precision]).contiguous()


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
@pytest.mark.parametrize("starting", [True, False])
@pytest.mark.parametrize("N", [37, 200])
def test_xn_input_matches_oracle(precision, starting, N):
    g = torch.Generator().manual_seed(300 + N)
    z = torch.randn(1, N, N, 128, generator=g)
    mask = rand_mask(g, 1, N)
    p = make_params(7, gate_bias=1.0)
    m = module(p, starting, precision)
    zc, mc = z.cuda(), mask.cuda()
    xn = _ln16(zc, m.layer_norm, starting, precision)
    y = m(zc, mc, xn=xn)
    ref = tri_attention_ref(z.double(), mask.double(), {k: (v.double() if v is not None else None) for k, v in p.items()},
                            starting=starting, dtype=torch.float64)
    assert_parity(y, ref, precision, "xn")
    # and close to the path that normalises z itself (the two LayerNorms round alike up to 1 ulp)
    y_plain = m(zc, mc)
    assert (y - y_plain).abs().max() < 1e-2


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
def test_keep_t_is_the_transposed_update(precision):
    N = 150
    g = torch.Generator().manual_seed(5)
    z = torch.randn(1, N, N, 128, generator=g).cuda()
    mask = rand_mask(g, 1, N).cuda()
    m = module(make_params(3, gate_bias=1.0), False, precision)
    y = m(z, mask)
    yt = m(z, mask, keep_t=True)
    assert torch.equal(yt, y.transpose(1, 2))


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
@pytest.mark.parametrize("starting", [True, False])
def test_f16_addln(precision, starting):
    N = 140
    g = torch.Generator().manual_seed(11)
    z = torch.randn(1, N, N, 128, generator=g).cuda()
    mask = rand_mask(g, 1, N).cuda()
    m = module(make_params(4, gate_bias=1.0), starting, precision)
    ln_next = torch.nn.LayerNorm(128).cuda()
    with torch.no_grad():
        ln_next.weight.copy_(1.0 + 0.1 * torch.randn(128, generator=g).cuda())
        ln_next.bias.copy_(0.1 * torch.randn(128, generator=g).cuda())
    xn = _ln16(z, m.layer_norm, starting, precision)
    z_new, ln_out = m.f16_addln(z, mask, xn, ln_next)
    # z_new: the residual update through the xn path
    assert torch.equal(z_new, z + m(z, mask, xn=xn))
    # ln_out: the next LayerNorm of z_new, fp32 statistics then one rounding to 16 bits
    ref = F.layer_norm(z_new, (128,), ln_next.weight, ln_next.bias, 1e-5)
    ulp = 2.0 ** -7 if precision == "bf16" else 2.0 ** -10
    assert ln_out.dtype == T16[precision]
    assert ((ln_out.float() - ref).abs() <= ulp * ref.abs() + 1e-3).all()
    # trans_out: the same values with the two N axes swapped; w_tb: the next tri bias from ln_out
    w_tb = 0.1 * torch.randn(4, 128, generator=g).cuda()
    z2, ln_t, tb = m.f16_addln(z, mask, xn, ln_next, trans_out=True, w_tb=w_tb)
    assert torch.equal(z2, z_new) and torch.equal(ln_t, ln_out.transpose(1, 2))
    # the next tri bias from the output kernel's epilogue (PAIRTB): fp32 sums of the rounded ln_out values,
    # one rounding to fp16, in ln_out's (here transposed) layout
    tb_ref = (ln_t.float() @ w_tb.t()).permute(0, 3, 1, 2)
    assert tb.shape == (1, 4, N, N) and tb.dtype == torch.float16
    assert ((tb.float() - tb_ref).abs() <= 2.0 ** -11 * tb_ref.abs() + 1e-5).all()


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
@pytest.mark.parametrize("starting", [True, False])
def test_producer_tri_bias_is_consumed(precision, starting):
    """tb given with xn (attention.py:128-147): the projection takes the producer's tri bias instead of
    its own dot.  The producer's fp16 tb of the same xn gives the same layer up to the bias rounding;
    a tb of zeros gives the layer without a tri bias."""
    N = 150
    g = torch.Generator().manual_seed(17)
    z = torch.randn(1, N, N, 128, generator=g).cuda()
    mask = rand_mask(g, 1, N).cuda()
    p = make_params(6, gate_bias=1.0)
    m = module(p, starting, precision)
    ln_next = torch.nn.LayerNorm(128).cuda()
    xn = _ln16(z, m.layer_norm, starting, precision)
    tb = (xn.float() @ m.linear.weight.detach().float().t()).permute(0, 3, 1, 2).to(torch.float16).contiguous()
    z_own, ln_own = m.f16_addln(z, mask, xn, ln_next)
    z_tb, ln_tb = m.f16_addln(z, mask, xn, ln_next, tb=tb)
    d = (z_tb - z_own).abs()
    assert float(d.max()) < 2e-2 and float(d.mean()) < 1e-3
    # with a zero tri bias the result is the layer without one (oracle with w_b = 0)
    p0 = dict(p, w_b=torch.zeros_like(p["w_b"]))
    z_0, _ = m.f16_addln(z, mask, xn, ln_next, tb=torch.zeros_like(tb))
    ref = tri_attention_ref(z.cpu().double(), mask.cpu().double(),
                            {k: (v.double() if v is not None else None) for k, v in p0.items()},
                            starting=starting, dtype=torch.float64)
    assert_parity(z_0 - z, ref, precision, "tb = 0")
    with pytest.raises(ValueError):
        m.f16_addln(z, mask, None, ln_next, tb=tb)


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
def test_tri_bias_handover_chain_matches_oracle(precision):
    """The reference's f16 pair block with the tri bias handed over (kernels.py:1537-1539): tri_mul_in
    -> (ln_start, tb_start) -> start layer on them -> (ln_end transposed, tb_end) -> end layer on them.
    Each layer's update is checked against the float64 oracle applied to that layer's actual input."""
    from boltz_mlx_b200 import TriangleMultiplicationIncoming, load_trimul_params
    from oracle.trimul_ref import make_params as tm_params, trimul_ref

    N = 128
    g = torch.Generator().manual_seed(29)
    z = torch.randn(1, N, N, 128, generator=g)
    mask = rand_mask(g, 1, N)
    pm, ps, pe = tm_params(31), make_params(32, gate_bias=1.0), make_params(33, gate_bias=1.0)
    tmi = load_trimul_params(TriangleMultiplicationIncoming(128, precision=precision).cuda(), pm)
    start, end = module(ps, True, precision), module(pe, False, precision)
    ln_last = torch.nn.LayerNorm(128).cuda()
    zc, mc = z.cuda(), mask.cuda()
    z1, xn1, tb1 = tmi.f16_addln(zc, mc, None, start.layer_norm, w_tb=start.tb_weight16())
    z2, xn2, tb2 = start.f16_addln(z1, mc, xn1, end.layer_norm, trans_out=True, tb=tb1, w_tb=end.tb_weight16())
    z3, _ = end.f16_addln(z2, mc, xn2, ln_last, tb=tb2)
    d = lambda p: {k: (v.double() if v is not None else None) for k, v in p.items()}
    m64 = mask.double()
    z1_64, z2_64 = z1.cpu().double(), z2.cpu().double()
    # the tri-mult layer to its own tolerance (max error relative to the largest output, mean absolute)
    from tests.test_gpu_trimul import assert_parity as assert_trimul_parity
    assert_trimul_parity(z1 - zc, trimul_ref(z.double(), m64, d(pm), outgoing=False, dtype=torch.float64), precision,
                         "tri_mul_in")
    assert_parity(z2 - z1, tri_attention_ref(z1_64, m64, d(ps), starting=True, dtype=torch.float64), precision,
                  "start layer on the handed-over xn, tb")
    assert_parity(z3 - z2, tri_attention_ref(z2_64, m64, d(pe), starting=False, dtype=torch.float64), precision,
                  "end layer on the handed-over xn, tb")


@pytest.mark.parametrize("precision", ["bf16", "fp16"])
def test_pair_block_chain_matches_oracle(precision):
    """The reference's f16 pair block (kernels.py:1535-1543): LN_start(z) -> start layer + residual +
    LN_end written transposed -> end layer on it + residual (+ the next LayerNorm)."""
    N = 128
    g = torch.Generator().manual_seed(23)
    z = torch.randn(1, N, N, 128, generator=g)
    mask = rand_mask(g, 1, N)
    ps, pe = make_params(8, gate_bias=1.0), make_params(9, gate_bias=1.0)
    start, end = module(ps, True, precision), module(pe, False, precision)
    zc, mc = z.cuda(), mask.cuda()
    xn0 = _ln16(zc, start.layer_norm, True, precision)
    z1, xn1 = start.f16_addln(zc, mc, xn0, end.layer_norm, trans_out=True)
    z2, _ = end.f16_addln(z1, mc, xn1, start.layer_norm, trans_out=False)
    d = lambda p: {k: (v.double() if v is not None else None) for k, v in p.items()}
    z64 = z.double()
    r1 = z64 + tri_attention_ref(z64, mask.double(), d(ps), starting=True, dtype=torch.float64)
    r2 = r1 + tri_attention_ref(r1, mask.double(), d(pe), starting=False, dtype=torch.float64)
    assert_parity(z2 - zc, r2 - z64, precision, "pair block")
