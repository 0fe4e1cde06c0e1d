"""CPU: the oracle (oracle/triattn_ref.py) against the committed golden fixtures and against its
independent float64 restatement, on the reference's test shapes and mask patterns."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.triattn_ref import (CONFIGS, make_inputs, make_params, metrics, token_mask, tri_attention_np64,
                                tri_attention_ref)

GOLDEN = Path(__file__).parent / "golden" / "triattn_golden.npz"


def golden_cases():
    d = np.load(GOLDEN)
    names = sorted({k[:-5] for k in d.files if k.endswith("_meta")})
    return d, names


def golden_params(d, pid):
    p = {k: torch.from_numpy(d[f"p{pid}_{k}"]) for k in ("ln_w", "ln_b", "w_q", "w_k", "w_v", "w_g", "w_b", "w_o")}
    p["g_b"] = torch.from_numpy(d[f"p{pid}_g_b"]) if f"p{pid}_g_b" in d.files else None
    return p


def golden_case(d, name):
    B, N, pid = (int(x) for x in d[f"{name}_meta"])
    z = torch.from_numpy(d[f"{name}_z"].astype(np.float32))
    m = torch.from_numpy(d[f"{name}_mask"].astype(np.float32)) if f"{name}_mask" in d.files else None
    return z, m, golden_params(d, pid)


@pytest.mark.parametrize("starting", [True, False])
def test_oracle_reproduces_golden(starting):
    d, names = golden_cases()
    assert len(names) >= 6
    for name in names:
        z, m, p = golden_case(d, name)
        ref = d[f"{name}_y_{'start' if starting else 'end'}"]
        y64 = tri_attention_ref(z, m, p, starting=starting, dtype=torch.float64).numpy()
        assert metrics(y64, ref)["max_rel"] <= 1e-6, name  # fixtures are float32-rounded float64
        y32 = tri_attention_ref(z, m, p, starting=starting).numpy()
        assert metrics(y32, ref)["max_rel"] <= 1e-5, name  # the fp32 tolerance of the CUDA fp32 mode


@pytest.mark.parametrize("N", [1, 2, 9, 17, 33, 37])
@pytest.mark.parametrize("starting", [True, False])
def test_torch_oracle_vs_numpy64(N, starting):
    g = torch.Generator().manual_seed(N)
    B = 2 if N < 20 else 1
    z = torch.randn(B, N, N, 128, generator=g)
    m = (torch.rand(B, N, N, generator=g) > 0.3).float()
    if N > 7:
        m[:, 3, :] = 0
        m[:, :, 5] = 0
    p = make_params(N, gate_bias=1.0, ln_identity=False)
    y64 = tri_attention_ref(z, m, p, starting=starting, dtype=torch.float64).numpy()
    ynp = tri_attention_np64(z.numpy(), m.numpy(), p, starting=starting)
    assert metrics(y64, ynp)["max_rel"] <= 1e-12


def test_fully_masked_row_is_uniform_mean():
    """fp32 rounding of -1e9 + logit makes a fully masked row attend uniformly (kernels.py:579-581)."""
    N = 12
    g = torch.Generator().manual_seed(3)
    z = torch.randn(1, N, N, 128, generator=g)
    m = torch.ones(1, N, N)
    m[0, 4, :] = 0
    p = make_params(5)
    # uniform attention == all logits equal: compare against a mask-free run with zeroed q/k/bias
    y = tri_attention_ref(z, m, p, rows=(4, 5))
    p0 = dict(p, w_q=torch.zeros_like(p["w_q"]), w_k=torch.zeros_like(p["w_k"]), w_b=torch.zeros_like(p["w_b"]))
    yu = tri_attention_ref(z, None, p0, rows=(4, 5))
    assert metrics(y.numpy(), yu.numpy())["max_rel"] <= 1e-6


def test_row_range_and_chunking_match_full():
    N = 21
    g = torch.Generator().manual_seed(9)
    z = torch.randn(1, N, N, 128, generator=g)
    m = (torch.rand(1, N, N, generator=g) > 0.2).float()
    p = make_params(9, gate_bias=1.0)
    for starting in (True, False):
        full = tri_attention_ref(z, m, p, starting=starting)
        ch = tri_attention_ref(z, m, p, starting=starting, chunk_rows=4)
        assert metrics(ch.numpy(), full.numpy())["max_rel"] <= 1e-6
        part = tri_attention_ref(z, m, p, starting=starting, rows=(5, 13))
        ref = full[:, 5:13] if starting else full[:, :, 5:13].transpose(1, 2)
        assert metrics(part.numpy(), ref.numpy())["max_rel"] <= 1e-6


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_row_ids_match_row_ranges(dtype):
    """The row-list selection (one LayerNorm / tri-bias pass, any rows in any order) equals the row-range
    path row by row, including a fully masked row."""
    N = 19
    g = torch.Generator().manual_seed(12)
    z = torch.randn(1, N, N, 128, generator=g)
    m = (torch.rand(1, N, N, generator=g) > 0.3).float()
    m[:, 6, :] = 0
    p = make_params(12, gate_bias=1.0, ln_identity=False)
    ids = [18, 0, 6, 7, 3]
    for starting in (True, False):
        sel = tri_attention_ref(z, m, p, starting=starting, dtype=dtype, row_ids=ids)
        assert sel.shape == (1, len(ids), N, 128)
        for i, a in enumerate(ids):
            one = tri_attention_ref(z, m, p, starting=starting, dtype=dtype, rows=(a, a + 1))
            assert metrics(sel[:, i:i + 1].numpy(), one.numpy())["max_rel"] <= (1e-6 if dtype == torch.float32 else 1e-13)


def test_ending_node_is_starting_node_on_transpose():
    N = 15
    g = torch.Generator().manual_seed(4)
    z = torch.randn(1, N, N, 128, generator=g)
    m = (torch.rand(1, N, N, generator=g) > 0.2).float()
    p = make_params(4)
    ye = tri_attention_ref(z, m, p, starting=False)
    ys = tri_attention_ref(z.transpose(1, 2), m.transpose(1, 2), p, starting=True).transpose(1, 2)
    assert torch.equal(ye, ys)


def test_config_inputs():
    for cid, c in CONFIGS.items():
        t = token_mask(c["N"], c["pad"], c["seed_z"])
        n_pad = int((t == 0).sum())
        if c["pad"] == "fixed38":
            assert n_pad == 38
        elif c["pad"] == "uniform15":
            assert 0 <= n_pad <= int(0.15 * c["N"])
        elif c["pad"] == "frac05":
            assert n_pad == round(0.05 * c["N"])
        else:
            assert n_pad == 0
    z, pm, p = make_inputs(0)
    assert z.shape == (1, 128, 128, 128) and pm.shape == (1, 128, 128)
    assert torch.all(p["g_b"] == 1.0)
