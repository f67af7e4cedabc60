"""Quantization at and next to half-integer quotients.

The kernels compute codes from the reciprocal product and decide values that
land within 2^-14 of a half-integer exactly (division-free residual test, IEEE
division only in the last ambiguous case).  Rows here are built so that many
quotients x/s are exactly k + 1/2 or within an ulp of it: the row peak is
chosen per row and the other entries are peak * (2k+1)/254 rounded to the
input dtype.  Codes and scales must equal the reference's quantize_reference
(numerics.py:29-46, IEEE division then rint) bit for bit.
"""

import numpy as np
import pytest
import torch

from oracle import reference_numpy as ref

pytestmark = pytest.mark.gpu


def tie_rows(rows, k, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    peaks = torch.cat([
        torch.tensor([127.0, 254.0, 63.5, 3.0, 1.0, 0.5, 1000.0, 2.0 ** -20, 448.0, 7.0]),
        torch.rand(rows, generator=g) * 100 + 0.01,
    ])[:rows]
    kk = torch.randint(-127, 127, (rows, k), generator=g).float()
    x = peaks[:, None] * (2 * kk + 1) / 254.0
    jitter = torch.randint(-2, 3, (rows, k), generator=g).float()
    x = x.to(dtype)
    if dtype != torch.float32:  # nudge some values by one unit in the last place
        raw = x.view(torch.int16).to(torch.int32)
        # values that flushed to zero (tiny peaks in f16) keep their bits: one
        # unit below +0 is a NaN pattern
        nudge = (torch.rand(rows, k, generator=g) < 0.2) & ((raw & 0x7FFF) >= 4)
        bits = raw + jitter.to(torch.int32) * nudge
        x = bits.to(torch.int16).view(dtype)
    x[:, 0] = peaks.to(dtype)
    x[:, 1] = -(peaks / 2).to(dtype)
    return x


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("k", [4096, 16384, 200])
def test_int8_ties_bit_exact(dtype, k):
    import m5kernels_b200 as m5

    x = tie_rows(64, k, dtype, seed=k)
    q, s = m5.quantize(x.cuda(), "int8")
    rq, rs = ref.quantize_reference(x.float().numpy(), "int8")
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fp8_ties_bit_exact(dtype):
    import m5kernels_b200 as m5

    x = tie_rows(64, 4096, dtype, seed=3)
    q, s = m5.quantize(x.cuda(), "fp8")
    rq, rs = ref.quantize_reference(x.float().numpy(), "fp8")
    np.testing.assert_array_equal(s.cpu().numpy(), rs)
    np.testing.assert_array_equal(q.cpu().numpy().view(np.uint8), rq.view(np.uint8))


@pytest.mark.parametrize("block", [0, 128])
def test_hadamard_prep_ties_match_oracle(block):
    """The register-resident prep kernel uses the same near-tie rule."""
    import m5kernels_b200 as m5
    from oracle import c_oracle as co

    k = 4096
    x = tie_rows(32, k, torch.bfloat16, seed=11)
    signs = torch.ones(k, dtype=torch.int8)
    if block:
        q, s = m5.hadamard_quantize(x.cuda(), block, signs.cuda(), "int8")
        o = co.row_prep(x, block=block, signs=signs)
    else:
        gamma, sc, sh = torch.ones(k), torch.zeros(k), torch.zeros(k)
        q, s = m5.fused_norm_hadamard_quantize(x.cuda(), gamma.cuda(), sc.cuda(), sh.cuda(),
                                               signs.cuda(), 64, norm="rms")
        o = co.row_prep(x, block=64, norm="rms", eps=1e-5, round_output=True, gamma=gamma,
                        scale=sc, shift=sh, signs=signs)
    assert torch.equal(q.cpu(), o["q"]) and torch.equal(s.cpu(), o["s"])

