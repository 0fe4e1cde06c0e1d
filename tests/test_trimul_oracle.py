"""CPU: the triangle-multiplication oracle (oracle/trimul_ref.py) against its independent float64
einsum formulation, on the reference tests' shapes (tiny and ragged N, B = 2, masked rows and
columns), both edge directions; channel blocking does not change the result."""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.trimul_ref import PARAM_SHAPES, make_params, trimul_np64, trimul_ref

GOLDEN = Path(__file__).parent / "golden" / "trimul_golden.npz"


def golden_cases():
    d = np.load(GOLDEN)
    return d, sorted({k[:-5] for k in d.files if k.endswith("_meta")})


def golden_case(d, name):
    B, N, pid = (int(x) for x in d[f"{name}_meta"])
    z = torch.from_numpy(d[f"{name}_z"].astype(np.float32))
    m = torch.from_numpy(d[f"{name}_mask"].astype(np.float32)) if f"{name}_mask" in d.files else None
    p = {k: torch.from_numpy(d[f"p{pid}_{k}"]) for k in PARAM_SHAPES}
    return z, m, p


def _inputs(B, N, seed):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(B, N, N, 128, generator=g)
    m = (torch.rand(B, N, N, generator=g) > 0.25).float()
    if N > 5:
        m[:, 2, :] = 0.0
        m[:, :, 4] = 0.0
    return z, m


@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("B,N", [(1, 1), (1, 5), (2, 9), (1, 33)])
def test_oracle_matches_float64_einsums(outgoing, B, N):
    z, m = _inputs(B, N, 100 + N)
    p = make_params(3)
    ref = trimul_ref(z, m, p, outgoing=outgoing, dtype=torch.float64).numpy()
    alt = trimul_np64(z.numpy(), m.numpy(), {k: v.numpy() for k, v in p.items()}, outgoing=outgoing)
    np.testing.assert_allclose(ref, alt, rtol=1e-10, atol=1e-10)
    f32 = trimul_ref(z, m, p, outgoing=outgoing).numpy()
    assert np.abs(f32 - alt).max() <= 1e-4 * max(1.0, np.abs(alt).max())


def test_channel_blocking_is_exact():
    z, m = _inputs(1, 17, 7)
    p = make_params(4)
    a = trimul_ref(z, m, p, outgoing=False, dtype=torch.float64, channel_block=128)
    b = trimul_ref(z, m, p, outgoing=False, dtype=torch.float64, channel_block=5)
    assert torch.allclose(a, b, rtol=1e-12, atol=1e-12)


def test_incoming_is_outgoing_on_the_transpose():
    """o_in[i,j] = sum_k a[k,i] b[k,j] is the outgoing product of the transposed pair tensor (the
    output gate reads the untransposed pair, so it is made constant here)."""
    z, m = _inputs(1, 11, 8)
    p = make_params(5)
    p["g_out"] = torch.zeros_like(p["g_out"])
    yin = trimul_ref(z, m, p, outgoing=False, dtype=torch.float64)
    yout_t = trimul_ref(z.transpose(1, 2), m.transpose(1, 2), p, outgoing=True, dtype=torch.float64)
    assert torch.allclose(yin, yout_t, rtol=1e-12, atol=1e-12)


def test_golden_fixtures_reproduce():
    """The committed fixtures (tests/golden/make_trimul_golden.py) are the oracle's float64 output stored
    in float32: the float64 oracle reproduces them to that rounding, the independent einsum form agrees,
    and the fp32 oracle stays within 1e-5 of them (the fp32 bar)."""
    d, names = golden_cases()
    assert len(names) == 5
    for name in names:
        z, m, p = golden_case(d, name)
        for outgoing, tag in ((True, "out"), (False, "in")):
            want = d[f"{name}_y_{tag}"].astype(np.float64)  # stored in float32
            got = trimul_ref(z.double(), None if m is None else m.double(), p, outgoing=outgoing,
                             dtype=torch.float64).numpy()
            np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)
            alt = trimul_np64(z.numpy(), None if m is None else m.numpy(), {k: v.numpy() for k, v in p.items()},
                              outgoing=outgoing)
            np.testing.assert_allclose(alt, want, rtol=1e-6, atol=1e-6)
            f32 = trimul_ref(z, m, p, outgoing=outgoing).numpy()
            assert np.abs(f32 - want).max() <= 1e-5 * max(1.0, np.abs(want).max()), name
