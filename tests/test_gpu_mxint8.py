"""GPU parity of the MXINT8 block quantization (quantize(x, "mxint8")).

Bar: codes and E8M0 exponent bytes bit-exact against the reference's own
golden vectors (bf16 rows, tests/golden/reference_vectors.npz) and against the
C restatement on bf16 / fp16 / fp32 rows with zero blocks, subnormal and huge
block peaks, ragged row counts and widths from one block to K = 16384.
"""

import numpy as np
import pytest
import torch

from oracle import c_oracle as co

pytestmark = pytest.mark.gpu

DEV = "cuda"


def test_mxint8_golden(golden):
    import m5kernels_b200 as m5

    xb = torch.from_numpy(golden["quant_x_bf16"].astype(np.int16)).view(torch.bfloat16)
    q, e = m5.quantize(xb.to(DEV), "mxint8")
    np.testing.assert_array_equal(q.cpu().numpy(), golden["quant_mxint8_q"])
    np.testing.assert_array_equal(e.cpu().numpy(), golden["quant_mxint8_s"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 32), (3, 64), (7, 5376), (129, 4096), (33, 16384)])
def test_mxint8_matches_restatement(dtype, shape):
    import m5kernels_b200 as m5

    rows, k = shape
    g = torch.Generator().manual_seed(rows * 7 + k)
    x = torch.randn(rows, k, generator=g)
    x[0, :32] = 0
    if rows > 2:
        x[1, k - 32:] *= 1e-6 if dtype == torch.float16 else 1e-39
        x[2, : min(64, k)] *= 1e4 if dtype == torch.float16 else 1e30
    x = x.to(dtype)
    q, e = m5.quantize(x.to(DEV), "mxint8")
    eq, ee = co.quantize_mxint8(x)
    assert torch.equal(q.cpu(), eq) and torch.equal(e.cpu(), ee)
