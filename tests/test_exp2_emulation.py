"""CPU emulation (float32, bit for bit) of the core kernel's MUFU-free exponential
(exp2_pair_poly_f16 in boltz_mlx_b200/csrc/kernels_tc.cu): y = max(x - m, -32), n = round(y) by the
1.5 * 2^23 shifter, f = y - n, 2^f by the fitted cubic, exponent-field add, then fp16 rounding."""

import numpy as np

C0 = np.float32(float.fromhex("0x1.fff696p-1"))
C1 = np.float32(float.fromhex("0x1.62f31ap-1"))
C2 = np.float32(float.fromhex("0x1.f0dd6ep-3"))
C3 = np.float32(float.fromhex("0x1.c3f60cp-5"))
SH = np.float32(12582912.0)


def exp2_poly(y):
    y = np.maximum(np.asarray(y, np.float32), np.float32(-32.0))
    t = (y + SH).astype(np.float32)
    n = (t - SH).astype(np.float32)
    f = (y - n).astype(np.float32)
    p = np.float32(C3) * f + C2  # fma in the kernel; float32 rounding differences are far below the bound
    p = (p * f + C1).astype(np.float32)
    p = (p * f + C0).astype(np.float32)
    with np.errstate(over="ignore"):  # the exponent-field add wraps modulo 2^32, as in the kernel
        bits = p.view(np.uint32) + (t.view(np.uint32) << np.uint32(23))
    return np.asarray(bits, np.uint32).view(np.float32)


def test_relative_error_over_the_used_range():
    y = np.linspace(-32.0, 8.0, 400001, dtype=np.float32)
    got = exp2_poly(y).astype(np.float64)
    ref = np.exp2(y.astype(np.float64))
    rel = np.abs(got - ref) / ref
    assert rel.max() < 1.0e-4, rel.max()
    # after the fp16 rounding of P the error is the fp16 half-ulp plus the fit error
    got16 = got.astype(np.float16).astype(np.float64)
    normal = ref > 2.0 ** -14
    assert (np.abs(got16 - ref) / ref)[normal].max() < 2.0 ** -11 + 1.0e-4


def test_masked_and_padded_logits_vanish():
    # mask bias (-1e9 log2 e) and padded keys (-1e30): clamped to -32, i.e. 2^-32, zero in fp16
    for y in (-1.4426950e9, -1e30, -40.0, -32.0):
        v = exp2_poly(np.float32(y))
        assert 0.0 <= v <= 2.0 ** -31
        assert np.float16(v) == 0.0
    assert exp2_poly(np.float32(0.0)) == np.float32(exp2_poly(np.float32(0.0)))
    assert abs(float(exp2_poly(np.float32(0.0))) - 1.0) < 1e-4
    assert abs(float(exp2_poly(np.float32(8.0))) - 256.0) < 256.0 * 1e-4
