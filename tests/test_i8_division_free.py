"""The INT8 codes of the quantization kernels come from a division-free
correctly rounded quotient (csrc/common.cuh, i8_pair_div): y = RN(1/s),
q = RN(x y), r = x - q s in one FMA, c = RN(q + r y) -- Markstein's
correction step.  The kernels rely on rint(c) == rint(RN(x / s)), the
reference's code (src/m5kernels/numerics.py:29-46), for every scale
s >= 2^-90 and |x| <= 127.0001 s.  These CPU checks (the C restatement in
oracle/m5_oracle.c) compare the two codes for every bf16 value against scales
of bf16 row peaks, scales with significands next to 1 and 2, the 2^-90 edge,
and random scales, plus fp32 values next to half-integer quotients.  The RMS
folding's codes, rint(RN(RN(v / peak) * 127)), need the corrected
quotient itself to equal RN(x / s) wherever a code can be nonzero
(|x / s| >= 2^-12), which the last test checks.  The GPU tests check the
kernels themselves against the IEEE-division oracle."""

import ctypes
import struct

import numpy as np

from oracle import c_oracle as co


def _scales():
    out = []
    for e in range(-20, 21, 3):  # s = amax / 127 for every bf16 peak mantissa
        for m in range(128):
            amax = np.float32((1.0 + m / 128.0) * 2.0 ** e)
            out.append(np.float32(amax / np.float32(127.0)))
    for e in (-90, -60, -1, 0, 1, 40, 99):  # significands next to 1 and 2
        for d in range(0, 64, 7):
            for frac in (d, 0x7FFFFF - d):
                out.append(struct.unpack("<f", struct.pack("<I", ((e + 127) << 23) | frac))[0])
    out.append(np.float32(2.0 ** -90))
    rng = np.random.default_rng(5)
    bits = ((rng.integers(37, 227, 400) << 23) | rng.integers(0, 1 << 23, 400)).astype(np.uint32)
    out.extend(bits.view(np.float32).tolist())
    return np.asarray(out, dtype=np.float32)


def test_bf16_codes_match_ieee_division():
    s = _scales()
    tested = ctypes.c_int64(0)
    bad = co.lib().m5o_check_i8_div_free(s.ctypes.data, s.size, ctypes.byref(tested))
    assert tested.value > 50_000_000
    assert bad == 0


def test_fp32_codes_match_ieee_division():
    tested = ctypes.c_int64(0)
    bad = co.lib().m5o_check_i8_div_free_f32(2_000_000, 11, ctypes.byref(tested))
    assert tested.value > 1_500_000
    assert bad == 0


def test_corrected_quotient_is_the_ieee_quotient():
    s = _scales()
    tested = ctypes.c_int64(0)
    bad = co.lib().m5o_check_div_free_quotient(s.ctypes.data, s.size, 2.0 ** -12, 448.5,
                                                2_000_000, 13, ctypes.byref(tested))
    assert tested.value > 10_000_000
    assert bad == 0
