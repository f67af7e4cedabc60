"""GPU parity of the grouped Q/K/V projection (weights in [head, stream, 128] order).

The reference's H3 integration runs one grouped INT8 projection whose output
columns are [head, stream (Q, K, V), channel] and writes three head-major BF16
tensors: Q and K with per-head RMSNorm (their own gammas) and split-half RoPE,
V as the rounded projection only (integrations/h3/qkv-candidate.md:30-43,
qkv_reference.h:15-36, docs/qk-rope-fusion.md:12).  Bars: every stream
bit-exact against the C restatement applied to exact INT32 accumulators, equal
to the separate single-projection path, and within 2 bf16 ulp (or relative L2
1e-3) of the float64 reference on decoded operands.
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


def _case(m, heads, k, half, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    x[0] = 0  # a zero row: Q/K outputs are exactly zero, V too
    x = x.to(torch.bfloat16)
    ws = [(torch.randn(heads * 128, k, generator=g) * k ** -0.5).to(torch.bfloat16)
          for _ in range(3)]
    gq = (1 + 0.2 * torch.randn(128, generator=g)).to(torch.bfloat16)
    gk = (1 + 0.2 * torch.randn(128, generator=g)).to(torch.bfloat16)
    ang = (torch.rand(m, half, generator=g) * 2 - 1) * np.pi
    return x, ws, gq, gk, torch.cos(ang).to(torch.bfloat16), torch.sin(ang).to(torch.bfloat16)


@pytest.mark.parametrize("m,heads,k,half", [(17, 1, 128, 48), (129, 3, 256, 48),
                                            (300, 5, 512, 64), (1000, 4, 1024, 33),
                                            (4096, 8, 512, 48), (520, 2, 2048, 8)])
def test_grouped_qkv_bit_exact(ops, m, heads, k, half):
    x, ws, gq, gk, cos, sin = _case(m, heads, k, half, seed=m + heads)
    w = ops.grouped_qkv_weights(*ws)
    aq, sa = ops.quantize(x.to(DEV), "int8")
    bq, sb = ops.quantize(w.to(DEV), "int8")
    q, kk, v = ops.projection_qkv_rope(aq, bq, gq.to(DEV), gk.to(DEV), cos.to(DEV), sin.to(DEV),
                                       "int8", a_scales=sa, b_scales=sb)
    assert all(tuple(t.shape) == (heads, m, 128) for t in (q, kk, v))
    acc = co.gemm_i8_acc_fast(aq.cpu(), bq.cpu()).view(m, heads, 3, 128)
    sbs = sb.cpu().view(heads, 3, 128)
    for stream, got, gamma in ((0, q, gq), (1, kk, gk)):
        a_s = acc[:, :, stream, :].reshape(m, heads * 128).float()
        expect = co.qk_rope_from_acc(a_s, sa.cpu(), sbs[:, stream].reshape(-1), gamma, cos, sin,
                                     half, 1e-5)
        assert torch.equal(got.cpu(), expect), f"stream {stream}"
    acc_v = acc[:, :, 2, :].reshape(m, heads * 128).contiguous()
    expect_v = co.gemm_epilogue(acc_v, sa.cpu(), sbs[:, 2].reshape(-1).contiguous())
    assert torch.equal(v.cpu(), expect_v.view(m, heads, 128).permute(1, 0, 2))
    assert torch.equal(q[:, 0].cpu(), torch.zeros(heads, 128, dtype=torch.bfloat16))
    assert torch.equal(v[:, 0].cpu(), torch.zeros(heads, 128, dtype=torch.bfloat16))


def test_grouped_equals_separate_projections_and_reference(ops):
    m, heads, k, half = 777, 4, 768, 48
    x, ws, gq, gk, cos, sin = _case(m, heads, k, half, seed=5)
    wd = [w.to(DEV) for w in ws]
    aq, sa = ops.quantize(x.to(DEV), "int8")
    codes = [ops.quantize(w, "int8") for w in wd]
    bq = ops.grouped_qkv_weights(*[c[0] for c in codes])
    sb = ops.grouped_qkv_weights(*[c[1].view(-1, 1) for c in codes]).view(-1)
    cd, sd = cos.to(DEV), sin.to(DEV)
    q, kk, v = ops.projection_qkv_rope(aq, bq, gq.to(DEV), gk.to(DEV), cd, sd, "int8",
                                       a_scales=sa, b_scales=sb)
    q1 = ops.projection_qk_rope(aq, codes[0][0], gq.to(DEV), cd, sd, "int8", a_scales=sa,
                                b_scales=codes[0][1])
    k1 = ops.projection_qk_rope(aq, codes[1][0], gk.to(DEV), cd, sd, "int8", a_scales=sa,
                                b_scales=codes[1][1])
    v1 = ops.gemm(aq, codes[2][0], "int8", a_scales=sa, b_scales=codes[2][1],
                  output_dtype=torch.bfloat16)
    assert torch.equal(q, q1) and torch.equal(kk, k1)
    assert torch.equal(v, v1.view(m, heads, 128).permute(1, 0, 2))
    # float64 reference (qkv_reference.h contract) on decoded operands
    dec_a = aq.cpu().double() * sa.cpu().double()[:, None]
    for out, (wq_, ws_), gamma in ((q, codes[0], gq), (kk, codes[1], gk)):
        dec = dec_a @ (wq_.cpu().double() * ws_.cpu().double()[:, None]).T
        r = ref.qk_rope_reference(dec.numpy().reshape(m, heads, 128), gamma.float().numpy(),
                                  cos.float().numpy(), sin.float().numpy(), epsilon=1e-5)["output"]
        yd = out.cpu().double().numpy()
        ulp = np.abs(yd - r) / np.maximum(np.abs(r) * 2.0**-7, 2.0**-133)
        assert ulp.max() <= 2 or ref.metrics(yd, r)["relative_l2"] <= 1e-3


def test_grouped_bf16_mode(ops):
    m, heads, k, half = 130, 2, 256, 64
    x, ws, gq, gk, cos, sin = _case(m, heads, k, half, seed=9)
    w = ops.grouped_qkv_weights(*ws)
    q, kk, v = ops.projection_qkv_rope(x.to(DEV), w.to(DEV), gq.to(DEV), gk.to(DEV),
                                       cos.to(DEV), sin.to(DEV), "bf16")
    dot = (x.double() @ w.double().T).view(m, heads, 3, 128)
    for out, s, gamma in ((q, 0, gq), (kk, 1, gk)):
        r = ref.qk_rope_reference(dot[:, :, s].numpy(), gamma.float().numpy(),
                                  cos.float().numpy(), sin.float().numpy())["output"]
        assert ref.metrics(out.cpu().double().numpy(), r)["relative_l2"] <= 1e-2
    rv = dot[:, :, 2].permute(1, 0, 2).numpy()
    assert ref.metrics(v.cpu().double().numpy(), rv)["relative_l2"] <= 1e-2


def test_grouped_contract(ops):
    a = torch.zeros(4, 128, dtype=torch.int8, device=DEV)
    b = torch.zeros(256, 128, dtype=torch.int8, device=DEV)
    g = torch.ones(128, dtype=torch.bfloat16, device=DEV)
    cs = torch.ones(4, 48, dtype=torch.bfloat16, device=DEV)
    sa = torch.ones(4, device=DEV)
    with pytest.raises(ValueError, match="heads, 3, 128"):
        ops.projection_qkv_rope(a, b, g, g, cs, cs, "int8", a_scales=sa,
                                b_scales=torch.ones(256, device=DEV))
    with pytest.raises(NotImplementedError, match="INT8 or BF16"):
        ops.projection_qkv_rope(a, b, g, g, cs, cs, "fp8")
