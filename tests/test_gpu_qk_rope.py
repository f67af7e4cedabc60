"""GPU parity of the fused Q/K projection + per-head RMSNorm + RoPE.

Bar: bit-exact against the C restatement of the epilogue applied to exact
INT32 accumulators (the fused path and a staged projection share one
integer dot and one FP32 order, as the reference requires with
tests/test_qk_rope_metal.py:78-81); within 2 bf16 ulp or relative L2 1e-3 of
the float64 reference qk_rope_reference on decoded operands.
"""

import numpy as np
import pytest
import torch

from oracle import c_oracle as co
from oracle import reference_numpy as ref

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    import m5kernels_b200 as m

    return m


def _inputs(m, n, k, half, seed=29):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(torch.bfloat16)
    gamma = (1 + 0.02 * torch.randn(128, generator=g)).to(torch.bfloat16)
    ang = (torch.rand(m, half, generator=g) * 2 - 1) * np.pi
    return x, w, gamma, torch.cos(ang).to(torch.bfloat16), torch.sin(ang).to(torch.bfloat16)


@pytest.mark.parametrize("shape,half", [((1, 128, 64), 64), ((17, 384, 96), 48),
                                        ((65, 256, 256), 64), ((129, 128, 64), 1),
                                        ((300, 512, 1024), 64), ((200, 256, 512), 33),
                                        # CTA-pair tiles of two heads: an odd head count
                                        # (last tile holds one head), and a last wave split
                                        # into half tiles, one of them past the last head
                                        ((512, 384, 256), 64), ((4096, 1408, 256), 64)])
def test_qk_rope_bit_exact_and_reference(ops, shape, half):
    m, n, k = shape
    x, w, gamma, cos, sin = _inputs(m, n, k, half)
    aq, sa = ops.quantize(x.to(DEV), "int8")
    bq, sb = ops.quantize(w.to(DEV), "int8")
    y = ops.projection_qk_rope(aq, bq, gamma.to(DEV), cos.to(DEV), sin.to(DEV), "int8",
                               a_scales=sa, b_scales=sb, epsilon=1e-5).cpu()
    acc = co.gemm_i8_acc(aq.cpu(), bq.cpu()).float()
    expect = co.qk_rope_from_acc(acc, sa.cpu(), sb.cpu(), gamma, cos, sin, half, 1e-5)
    assert torch.equal(y, expect)
    # staged path: the same projection materialized in BF16 then post-processed
    proj = ops.gemm(aq, bq, "int8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16).cpu()
    staged = co.qk_rope_from_acc(proj.float(), None, None, gamma, cos, sin, half, 1e-5)
    assert torch.equal(y, staged)
    # float64 reference on decoded operands
    dec = (aq.cpu().double() * sa.cpu().double()[:, None]) @ (bq.cpu().double() * sb.cpu().double()[:, None]).T
    r = ref.qk_rope_reference(dec.numpy().reshape(m, n // 128, 128), gamma.float().numpy(),
                              cos.float().numpy(), sin.float().numpy(), epsilon=1e-5)["output"]
    yd = y.double().numpy()
    ulp = np.abs(yd - r) / np.maximum(np.abs(r) * 2.0**-7, 2.0**-133)
    assert ulp.max() <= 2 or ref.metrics(yd, r)["relative_l2"] <= 1e-3


def test_qk_rope_bf16_mode(ops):
    m, n, k = 130, 256, 256
    x, w, gamma, cos, sin = _inputs(m, n, k, 64)
    y = ops.projection_qk_rope(x.to(DEV), w.to(DEV), gamma.to(DEV), cos.to(DEV), sin.to(DEV),
                               "bf16").cpu()
    dot = x.double() @ w.double().T
    r = ref.qk_rope_reference(dot.numpy().reshape(m, 2, 128), gamma.float().numpy(),
                              cos.float().numpy(), sin.float().numpy())["output"]
    assert ref.metrics(y.double().numpy(), r)["relative_l2"] <= 1e-2


def test_qk_rope_pairing_direction(ops):
    """Split-half pairing: with cos=0, sin=1, out[:R] = -u[R:2R], out[R:2R] = u[:R]."""
    m, n, k, half = 4, 128, 128, 2
    aq = torch.zeros(m, k, dtype=torch.int8)
    bq = torch.zeros(n, k, dtype=torch.int8)
    for j in range(6):
        bq[j, j] = j + 1
    aq[:, :6] = 1
    sa = torch.ones(m)
    sb = torch.ones(n)
    gamma = torch.ones(128, dtype=torch.bfloat16)
    cos = torch.zeros(m, half, dtype=torch.bfloat16)
    sin = torch.ones(m, half, dtype=torch.bfloat16)
    y = ops.projection_qk_rope(aq.to(DEV), bq.to(DEV), gamma.to(DEV), cos.to(DEV), sin.to(DEV),
                               "int8", a_scales=sa.to(DEV), b_scales=sb.to(DEV)).cpu()[0, 0, :6].float()
    inv = 1 / np.sqrt((1 + 4 + 9 + 16 + 25 + 36) / 128 + 1e-5)
    np.testing.assert_allclose(y.numpy(), np.array([-3, -4, 1, 2, 5, 6]) * inv, rtol=1e-2)


def test_qk_rejections(ops):
    aq = torch.zeros(4, 64, dtype=torch.int8, device=DEV)
    bq = torch.zeros(100, 64, dtype=torch.int8, device=DEV)
    s = torch.ones(4, device=DEV)
    gamma = torch.ones(128, dtype=torch.bfloat16, device=DEV)
    cs = torch.ones(4, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError, match="128-wide heads"):
        ops.projection_qk_rope(aq, bq, gamma, cs, cs, a_scales=s, b_scales=torch.ones(100, device=DEV))
    with pytest.raises(NotImplementedError):
        ops.projection_qk_rope(aq, bq, gamma, cs, cs, "fp8")


@pytest.mark.parametrize("shape", [(256, 4096, 4096), (300, 512, 8192), (700, 1408, 4096)])
def test_qk_rope_splitk_bit_exact(ops, shape, monkeypatch):
    """Q/K projections with few rows take the split-K schedule (2 to 4 CTA
    pairs per tile; an odd head count and an M tail): the finishing pair adds
    the INT32 partial sums before the BF16 projection, so the output is
    bit-identical to the C epilogue and to the data-parallel schedule."""
    from m5kernels_b200 import _lib

    m, n, k = shape
    half = 64
    assert int(_lib.lib().m5b_gemm_workspace_bytes(m, n, k, _lib.MODE["int8"])) > 0
    x, w, gamma, cos, sin = _inputs(m, n, k, half, seed=61)
    aq, sa = ops.quantize(x.to(DEV), "int8")
    bq, sb = ops.quantize(w.to(DEV), "int8")
    args = (aq, bq, gamma.to(DEV), cos.to(DEV), sin.to(DEV), "int8")
    y = ops.projection_qk_rope(*args, a_scales=sa, b_scales=sb, epsilon=1e-5)
    y2 = ops.projection_qk_rope(*args, a_scales=sa, b_scales=sb, epsilon=1e-5)
    acc = co.gemm_i8_acc_fast(aq.cpu(), bq.cpu()).float()
    expect = co.qk_rope_from_acc(acc, sa.cpu(), sb.cpu(), gamma, cos, sin, half, 1e-5)
    assert torch.equal(y.cpu(), expect) and torch.equal(y2, y)
    monkeypatch.setenv("M5B_GEMM_SPLITK", "0")
    dp = ops.projection_qk_rope(*args, a_scales=sa, b_scales=sb, epsilon=1e-5)
    assert torch.equal(dp, y)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("shape", [(512, 4096, 4096), (600, 1408, 8192)])
def test_qk_rope_cluster_splitk_bit_exact(ops, shape):
    """The cluster split-K schedule (two CTA pairs per tile in one 4-CTA
    cluster, partial sums through shared memory) under the Q/K epilogue:
    bit-identical to the C epilogue and to the data-parallel schedule."""
    from m5kernels_b200 import _lib

    m, n, k = shape
    half = 64
    x, w, gamma, cos, sin = _inputs(m, n, k, half, seed=67)
    aq, sa = ops.quantize(x.to(DEV), "int8")
    bq, sb = ops.quantize(w.to(DEV), "int8")
    args = (aq, bq, gamma.to(DEV), cos.to(DEV), sin.to(DEV), "int8")
    with ops.gemm_schedule(2, 0):
        y = ops.projection_qk_rope(*args, a_scales=sa, b_scales=sb, epsilon=1e-5)
    acc = co.gemm_i8_acc_fast(aq.cpu(), bq.cpu()).float()
    expect = co.qk_rope_from_acc(acc, sa.cpu(), sb.cpu(), gamma, cos, sin, half, 1e-5)
    assert torch.equal(y.cpu(), expect)
    with ops.gemm_schedule(0, 0):
        dp = ops.projection_qk_rope(*args, a_scales=sa, b_scales=sb, epsilon=1e-5)
    assert torch.equal(dp, y)
    assert _lib.device_status() == 0
