"""GPU: config 3 — a 128-layer start+end stack (64 blocks, distinct seeded weights, residual adds,
N=768, fp16) against the same stack through the library's fp32 path, which the parity tests pin to the
oracle at max_rel <= 1e-5 per layer.  The 16-bit error of every layer stays bounded instead of
compounding: the final z and the accumulated update both track the fp32 stack."""

import pytest

import bench

pytestmark = pytest.mark.gpu


def test_config3_stack_drift():
    r = bench.stack_drift(3, steps=1, warmup=1)
    print(r)
    assert r["layers"] == 128
    # measured on B200: max_rel 1.2e-3, mean_abs 4.5e-3 (update mean |.| 4.8), cos 0.9999996; bounds ~3-4x
    assert r["z"]["cos"] > 0.99999, r
    assert r["update"]["cos"] > 0.99999, r
    assert r["z"]["max_rel"] < 5e-3, r
    assert r["z"]["mean_abs"] < 3e-3 * r["update_abs_mean"] + 1e-3, r
