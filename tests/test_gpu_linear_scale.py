"""m5b_linear (online quantization -> W8A8 GEMM in one call) at scale.

The one-call projection must equal the two calls it stands for (quantize,
then gemm) bit for bit -- for partial 256-row blocks, zero rows, rows with
many exact half-integer quotients (a row peak of 127 * 2^e), every output
dtype, and on repeated calls that reuse the cached workspace.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _two_step(m5, x, wq, ws, out_dtype):
    q, s = m5.quantize(x, "int8")
    return m5.gemm(q, wq, "int8", a_scales=s, b_scales=ws, output_dtype=out_dtype)


def _acts(m, k, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x[m // 5] = 0.0
    # rows whose peak is 127 * 2^e: x / s lands exactly on half-integers
    x[m // 3, 0] = 127.0
    x[m // 3, 1:] = torch.randint(-254, 255, (k - 1,), generator=g).float() / 2.0
    x[m // 2, 0] = 63.5
    return x.to(torch.bfloat16)


SHAPES = [(256, 256, 64), (300, 520, 1024), (513, 384, 2048), (1000, 2048, 16384),
          (4096, 1024, 4160)]


@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{n}x{k}" for m, n, k in SHAPES])
def test_fused_linear_equals_two_launches(shape):
    import m5kernels_b200 as m5

    m, n, k = shape
    x = _acts(m, k, seed=m + k).to(DEV)
    g = torch.Generator().manual_seed(n)
    w = (0.02 * torch.randn(n, k, generator=g)).to(torch.bfloat16).to(DEV)
    wq, ws = m5.quantize(w, "int8")
    got = m5.linear(x, wq, ws, "int8")
    assert torch.equal(got, _two_step(m5, x, wq, ws, torch.bfloat16))


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_fused_linear_output_dtypes(out_dtype):
    import m5kernels_b200 as m5

    x = _acts(700, 3072, seed=3).to(DEV)
    w = (0.02 * torch.randn(640, 3072, generator=torch.Generator().manual_seed(4)))
    wq, ws = m5.quantize(w.to(torch.bfloat16).to(DEV), "int8")
    got = m5.linear(x, wq, ws, "int8", output_dtype=out_dtype)
    assert torch.equal(got, _two_step(m5, x, wq, ws, out_dtype))


def test_fused_linear_repeated_calls_reuse_the_workspace():
    import m5kernels_b200 as m5

    m, n, k = 2048, 1024, 8192
    g = torch.Generator().manual_seed(12)
    w = (0.02 * torch.randn(n, k, generator=g)).to(torch.bfloat16).to(DEV)
    wq, ws = m5.quantize(w, "int8")
    xs = [_acts(m, k, seed=s).to(DEV) for s in (21, 22, 23)]
    outs = [m5.linear(x, wq, ws, "int8") for x in xs]  # back to back, one workspace
    for x, y in zip(xs, outs):
        assert torch.equal(y, _two_step(m5, x, wq, ws, torch.bfloat16))
    assert m5._lib.device_status() == 0
