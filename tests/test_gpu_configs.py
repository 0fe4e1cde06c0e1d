"""GPU: parity at the benchmark configurations themselves (config 1: N=384 fp16, config 2: N=1024 bf16,
config 4: N=2048 bf16), for the start+end pair the bench times.

Two checks per configuration and node:
  * the WHOLE output tensor of the 16-bit layer against the library's fp32 layer on the same input
    (the fp32 path is pinned to the CPU oracle at max_rel <= 1e-5 by test_gpu_parity.py), with the
    north-star tolerance of a 16-bit layer against the fp32 reference: max_abs <= 2e-2, mean_abs <= 5e-3;
  * at least 64 attention rows of the 16-bit layer against the CPU oracle directly: rows spread over
    [0, N) with every residue modulo 4 (the attention core groups rows in 2s and 4s), plus the first
    and last rows and both sides of the padding boundary.  Every row covers every query tile.

The ending node runs on the starting node's fp32 output, as in the pair (z1 = z + start(z))."""

import pytest
import torch

from oracle.triattn_ref import make_inputs, make_params, tri_attention_ref
from tests._util import H16_MAX_ABS, H16_MEAN_ABS, assert_parity, module

pytestmark = pytest.mark.gpu

CFG_PRECISION = {1: "fp16", 2: "bf16", 4: "bf16"}


def sample_rows(N: int, n_pad: int, n: int = 64) -> list:
    rows = {min(N - 1, (i * N) // n + (i % 4)) for i in range(n)}
    rows |= {0, 1, 2, 3, N - 1, N // 2}
    if n_pad:
        rows |= {N - n_pad - 1, N - n_pad, N - n_pad + 1}
    return sorted(r for r in rows if 0 <= r < N)


def gpu_metrics(a: torch.Tensor, b: torch.Tensor) -> dict:
    d = (a - b).abs()
    return {"max_abs": float(d.max()), "mean_abs": float(d.double().mean()),
            "ref_absmax": float(b.abs().max()), "finite": bool(torch.isfinite(a).all())}


@pytest.mark.parametrize("cfg", [1, 2, 4])
def test_config_layers_whole_tensor_vs_fp32_path(cfg):
    z, pm, ps = make_inputs(cfg)
    pe = make_params(100 + cfg, gate_bias=1.0)
    prec = CFG_PRECISION[cfg]
    zc, mc = z.cuda(), pm.cuda()
    with torch.no_grad():
        for starting, p in ((True, ps), (False, pe)):
            m32 = module(p, starting, "fp32")
            y32 = m32(zc, mc)
            del m32
            m16 = module(p, starting, prec)
            y16 = m16(zc, mc)
            del m16
            torch.cuda.synchronize()
            m = gpu_metrics(y16, y32)
            assert m["finite"], f"cfg{cfg} start={starting}: non-finite output"
            assert m["max_abs"] <= H16_MAX_ABS and m["mean_abs"] <= H16_MEAN_ABS, f"cfg{cfg} start={starting}: {m}"
            if starting:
                zc = zc + y32  # the ending node's input: the pair's z1 (fp32 path)
            del y16, y32
            torch.cuda.empty_cache()


@pytest.mark.parametrize("cfg", [1, 2, 4])
def test_config_rows_vs_oracle(cfg):
    z, pm, ps = make_inputs(cfg)
    pe = make_params(100 + cfg, gate_bias=1.0)
    prec = CFG_PRECISION[cfg]
    N = z.shape[1]
    n_pad = int((pm[0, 0] == 0).sum())
    rows = sample_rows(N, n_pad)
    assert len(rows) >= 64
    zc, mc = z.cuda(), pm.cuda()
    for starting, p in ((True, ps), (False, pe)):
        y = module(p, starting, prec)(zc, mc)
        ya = (y if starting else y.transpose(1, 2))[:, rows].cpu()
        del y
        ref = tri_attention_ref(z, pm, p, starting=starting, row_ids=rows)
        assert_parity(ya, ref, prec, f"cfg{cfg} start={starting} {len(rows)} rows")
        if starting:
            # ending-node input: the pair's z1, through the fp32 path on the GPU (pinned to the oracle)
            z = z + module(p, True, "fp32")(zc, mc).cpu()
            zc = z.cuda()
        torch.cuda.empty_cache()
