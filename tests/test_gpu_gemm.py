"""GPU parity of the tcgen05 GEMM and its fused epilogues.

Bar: INT32 accumulators bit-exact (exact integer dot products); INT8 BF16 /
FP16 / FP32 outputs bit-exact against the C epilogue restatement
((float(acc) * sa) * sb, then bias or gate, then RNE) and, as the stated
bar, every BF16 output within 2 bf16 ulp of the float64 value (FP16 / FP32
outputs: relative L2 <= 1e-3); FP8 within relative L2 5e-3 of the float64
decoded dot; BF16 GEMM within relative L2 1e-5.
Shapes cover the reference's tail cases (tests/test_metal.py:28-53,
tests/test_qk_rope_metal.py:39-52): M, N and K not multiples of the tile.  A
K whose rows are not whole 16-byte TMA strides is refused (padding is not
implicit); those cases pad K explicitly with zero codes, as a caller must.
GEMMs with few rows take the split-K schedule (several CTA pairs per tile,
INT32 partial sums added by the last to finish); its outputs are checked
against the same oracle and against the data-parallel schedule
(M5B_GEMM_SPLITK=0) on tail shapes.
"""

import numpy as np
import pytest
import torch

from oracle import c_oracle as co
from oracle import reference_numpy as ref

pytestmark = pytest.mark.gpu

DEV = "cuda"
TAIL_SHAPES = [(1, 33, 64), (127, 65, 96), (65, 17, 257), (129, 128, 33), (17, 384, 96),
               (300, 520, 1024), (512, 2048, 2048)]


@pytest.fixture(scope="module")
def ops():
    import m5kernels_b200 as m

    return m


def _operands(m, n, k, seed=5, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g).to(dtype)
    b = (torch.randn(n, k, generator=g) * 0.02).to(dtype)
    return a, b


def _q(ops, t, mode="int8"):
    q, s = ops.quantize(t.to(DEV), mode)
    return q, s


def _pad16(q):
    """Explicit zero padding of int8 codes to a multiple of 16 per row (zero
    codes leave every dot product unchanged)."""
    k = q.shape[1]
    if k % 16 == 0:
        return q
    out = torch.zeros((q.shape[0], k + (-k) % 16), dtype=q.dtype, device=q.device)
    out[:, :k] = q
    return out


def _within_ulps(y, ref64, mant_bits, ulps=2):
    """Every element of y within `ulps` units in the last place (of a format with
    mant_bits explicit mantissa bits) of the float64 reference."""
    r = ref64.abs().clamp_min(2.0 ** -126)
    ulp = torch.exp2(torch.floor(torch.log2(r)) - mant_bits)
    return bool(((y.double() - ref64).abs() <= ulps * ulp).all())


@pytest.mark.parametrize("shape", TAIL_SHAPES)
def test_int8_accumulators_bit_exact(ops, shape):
    m, n, k = shape
    a, b = _operands(m, n, k)
    aq, _ = _q(ops, a)
    bq, _ = _q(ops, b)
    acc = ops.gemm(_pad16(aq), _pad16(bq), "int8", output_dtype=torch.int32).cpu()
    expect = co.gemm_i8_acc(aq.cpu(), bq.cpu())
    assert torch.equal(acc, expect)


@pytest.mark.parametrize("shape", TAIL_SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_int8_scaled_epilogue_bit_exact(ops, shape, out_dtype):
    m, n, k = shape
    a, b = _operands(m, n, k)
    aq, sa = _q(ops, a)
    bq, sb = _q(ops, b)
    y = ops.gemm(_pad16(aq), _pad16(bq), "int8", a_scales=sa, b_scales=sb,
                 output_dtype=out_dtype).cpu()
    acc = co.gemm_i8_acc(aq.cpu(), bq.cpu())
    expect = co.gemm_epilogue(acc, sa.cpu(), sb.cpu(), out_dtype=out_dtype)
    assert torch.equal(y, expect)
    # the stated bar against the float64 value of the decoded dot, sa*sb*acc
    # from the exact integer sums (summing decoded products in float64 instead
    # leaves rounding noise, e.g. 7e-17 where the exact dot is 0): BF16 within
    # 2 bf16 ulp elementwise, other outputs relative L2 <= 1e-3
    dec = acc.double() * sa.cpu().double()[:, None] * sb.cpu().double()[None, :]
    if out_dtype == torch.bfloat16:
        assert _within_ulps(y, dec, 7)
    else:
        assert ref.metrics(y.double().numpy(), dec.numpy())["relative_l2"] <= 1e-3


def test_ragged_k_is_refused_without_padding(ops):
    aq, sa = _q(ops, torch.ones(4, 33))
    with pytest.raises(NotImplementedError, match="padding is not implicit"):
        ops.gemm(aq, aq, "int8", a_scales=sa, b_scales=sa)


# few rows: split-K for INT8 when the 256 x 256 pair tiles fill at most a
# quarter of the CTA pairs (2 to 4 pairs per tile; M / N / K tails), else
# data-parallel with N-halves
SMALL_M_SHAPES = [(512, 4096, 16384), (256, 512, 4096), (1000, 1000, 3000), (768, 2048, 8192),
                  (300, 520, 1024), (512, 4096, 2048)]


@pytest.mark.parametrize("shape", SMALL_M_SHAPES)
@pytest.mark.parametrize("mode", ["int8", "fp8"])
def test_small_m_gemm(ops, shape, mode, monkeypatch):
    """GEMMs with few rows (a token-sharded rank's share, tiny problems): INT8
    accumulators and epilogue bit-exact, on split-K where it applies and
    identical to the data-parallel schedule, two calls in a row; FP8 within
    its bar."""
    from m5kernels_b200 import _lib

    m, n, k = shape
    a, b = _operands(m, n, k, seed=43)
    aq, sa = _q(ops, a, mode)
    bq, sb = _q(ops, b, mode)
    if mode == "fp8":
        if k % 128:
            return
        y = ops.gemm(aq, bq, "fp8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16).cpu()
        da = ref.dequantize(aq.cpu().numpy(), sa.cpu().numpy(), "fp8").astype(np.float64)
        db = ref.dequantize(bq.cpu().numpy(), sb.cpu().numpy(), "fp8").astype(np.float64)
        assert ref.metrics(y.float().numpy(), da @ db.T)["relative_l2"] <= 5e-3
        return
    expect = co.gemm_i8_acc_fast(aq.cpu(), bq.cpu())
    aq, bq = _pad16(aq), _pad16(bq)
    import os

    splitk = int(_lib.lib().m5b_gemm_workspace_bytes(m, n, aq.shape[1], _lib.MODE["int8"])) > 0
    if "M5B_GEMM_SPLITK" not in os.environ:  # the default rule
        assert splitk == (shape in ((256, 512, 4096), (1000, 1000, 3000)))
    for _ in range(2):
        acc = ops.gemm(aq, bq, "int8", output_dtype=torch.int32).cpu()
        assert torch.equal(acc, expect)
        y = ops.gemm(aq, bq, "int8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16)
        assert torch.equal(y.cpu(), co.gemm_epilogue(expect, sa.cpu(), sb.cpu()))
    monkeypatch.setenv("M5B_GEMM_SPLITK", "0")
    dp = ops.gemm(aq, bq, "int8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16)
    assert torch.equal(dp, y)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("shape", [(512, 2048, 2048), (256, 512, 4096), (1000, 1000, 3000),
                                   (4096, 4096, 4096)])
def test_every_schedule_gives_the_same_output(ops, shape):
    """The tune twin's schedules (split-K factors, raster groups) change only
    the time: outputs are bit-identical to the C epilogue under each of them,
    and the workspace size follows the schedule."""
    from m5kernels_b200 import _lib, cli

    m, n, k = shape
    a, b = _operands(m, n, k, seed=47)
    aq, sa = _q(ops, a)
    bq, sb = _q(ops, b)
    expect = co.gemm_epilogue(co.gemm_i8_acc_fast(aq.cpu(), bq.cpu()), sa.cpu(), sb.cpu())
    aq, bq = _pad16(aq), _pad16(bq)  # explicit zero codes: whole 16-byte TMA strides
    k = aq.shape[1]
    lib = _lib.lib()
    ws_default = lib.m5b_gemm_workspace_bytes(m, n, k, _lib.MODE["int8"])
    for split_k, group_m in cli.SCHEDULES:
        with ops.gemm_schedule(split_k, group_m):
            ws = lib.m5b_gemm_workspace_bytes(m, n, k, _lib.MODE["int8"])
            if split_k == 0:
                assert ws == 0
            y = ops.gemm(aq, bq, "int8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16)
        assert torch.equal(y.cpu(), expect), (split_k, group_m)
    # leaving the block restores the library's rule
    assert lib.m5b_gemm_workspace_bytes(m, n, k, _lib.MODE["int8"]) == ws_default
    assert _lib.device_status() == 0


def test_c1_config_w8a8(ops):
    """A [512,2048] ~N(0,1), W [2048,2048] ~N(0,0.02), seed 0."""
    g = torch.Generator().manual_seed(0)
    a = torch.randn(512, 2048, generator=g).to(torch.bfloat16)
    w = (torch.randn(2048, 2048, generator=g) * 0.02).to(torch.bfloat16)
    aq, sa = _q(ops, a)
    wq, sw = _q(ops, w)
    y = ops.gemm(aq, wq, "int8", a_scales=sa, b_scales=sw, output_dtype=torch.bfloat16).cpu()
    expect = co.gemm_epilogue(co.gemm_i8_acc_fast(aq.cpu(), wq.cpu()), sa.cpu(), sw.cpu())
    assert torch.equal(y, expect)


@pytest.mark.parametrize("table", [False, True])
def test_int8_bias_epilogue(ops, table):
    m, n, k = 200, 384, 512
    a, b = _operands(m, n, k, seed=7)
    aq, sa = _q(ops, a)
    bq, sb = _q(ops, b)
    g = torch.Generator().manual_seed(8)
    bias = torch.randn(3, n, generator=g) if table else torch.randn(n, generator=g)
    brm = (torch.arange(m, dtype=torch.int32) % 3) if table else None
    y = ops.gemm(aq, bq, "int8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16,
                 bias=bias.to(DEV), bias_row_map=brm.to(DEV) if table else None).cpu()
    acc = co.gemm_i8_acc(aq.cpu(), bq.cpu())
    expect = co.gemm_epilogue(acc, sa.cpu(), sb.cpu(), epi="bias_table" if table else "bias_vec",
                              bias=bias, bias_row_map=brm)
    assert torch.equal(y, expect)


@pytest.mark.parametrize("table", [False, True])
def test_int8_gated_epilogue_equals_staged(ops, table):
    m, n, k = 130, 256, 384
    a, b = _operands(m, n, k, seed=9)
    aq, sa = _q(ops, a)
    bq, sb = _q(ops, b)
    g = torch.Generator().manual_seed(10)
    residual = torch.randn(m, n, generator=g).to(torch.bfloat16)
    gate = (0.1 * torch.randn(2, n, generator=g)).to(torch.bfloat16)
    gate = gate if table else gate[0]
    grm = (torch.arange(m, dtype=torch.int32) // 65) if table else None
    y = ops.gemm(aq, bq, "int8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16,
                 residual=residual.to(DEV), gate=gate.to(DEV),
                 gate_row_map=grm.to(DEV) if table else None).cpu()
    acc = co.gemm_i8_acc(aq.cpu(), bq.cpu())
    expect = co.gemm_epilogue(acc, sa.cpu(), sb.cpu(), epi="gate_table" if table else "gate_vec",
                              residual=residual, gate=gate, gate_row_map=grm)
    assert torch.equal(y, expect)
    # staged: bf16 branch output, then the gated update (reference chain semantics)
    branch = ops.gemm(aq, bq, "int8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16).cpu()
    gsel = gate[grm.long()] if table else gate[None, :]
    staged = torch.addcmul(residual.float(), branch.float(), gsel.float()).to(torch.bfloat16)
    assert torch.equal(y, staged)


@pytest.mark.parametrize("shape", [(65, 33, 256), (300, 520, 1024), (256, 4096, 4096)])
def test_fp8_gemm_tolerance(ops, shape):
    m, n, k = shape
    a, b = _operands(m, n, k, seed=11)
    aq, sa = _q(ops, a, "fp8")
    bq, sb = _q(ops, b, "fp8")
    y = ops.gemm(aq, bq, "fp8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16).cpu()
    da = ref.dequantize(aq.cpu().numpy(), sa.cpu().numpy(), "fp8").astype(np.float64)
    db = ref.dequantize(bq.cpu().numpy(), sb.cpu().numpy(), "fp8").astype(np.float64)
    assert ref.metrics(y.float().numpy(), da @ db.T)["relative_l2"] <= 5e-3


def test_fp8_full_misaligned_output_tail(ops):
    a = torch.ones(65, 256, device=DEV)
    b = torch.ones(33, 256, device=DEV)
    aq, sa = ops.quantize(a, "fp8")
    bq, sb = ops.quantize(b, "fp8")
    y = ops.gemm(aq, bq, "fp8", a_scales=sa, b_scales=sb).cpu()
    torch.testing.assert_close(y, torch.full((65, 33), 256.0), rtol=1e-5, atol=0)


@pytest.mark.parametrize("mode", ["bf16", "fp16"])
@pytest.mark.parametrize("shape", [(1, 33, 64), (127, 65, 96), (300, 520, 1024)])
def test_float_gemm_tolerance(ops, mode, shape):
    m, n, k = shape
    dt = torch.bfloat16 if mode == "bf16" else torch.float16
    a, b = _operands(m, n, k, seed=12, dtype=dt)
    y = ops.gemm(a.to(DEV), b.to(DEV), mode, output_dtype=torch.float32).cpu()
    expect = a.double() @ b.double().T
    assert ref.metrics(y.numpy(), expect.numpy())["relative_l2"] <= 1e-5


def test_gemm_contract_rejections(ops):
    a = torch.ones(2, 96, device=DEV)
    b = torch.ones(3, 96, device=DEV)
    aq, sa = ops.quantize(a, "fp8")
    bq, sb = ops.quantize(b, "fp8")
    with pytest.raises(NotImplementedError, match="stride"):
        ops.gemm(aq, bq, "fp8", a_scales=sa, b_scales=sb)
    qa, qsa = ops.quantize(torch.ones(4, 64, device=DEV), "int8")
    with pytest.raises(ValueError, match="scales"):
        ops.gemm(qa, qa, "int8")
    with pytest.raises(NotImplementedError, match="BF16 output"):
        ops.gemm(qa, qa, "int8", a_scales=qsa, b_scales=qsa, residual=torch.zeros(4, 4, device=DEV),
                 gate=torch.zeros(4, device=DEV, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="K mismatch"):
        ops.gemm(qa, qa[:, :32], "int8", a_scales=qsa, b_scales=qsa)


@pytest.mark.parametrize("shape", [(4096, 4096, 256), (4000, 4000, 384), (9914, 4096, 128),
                                   (2304, 8448, 128)])
def test_pair_split_tail_bit_exact(ops, shape):
    """Shapes whose last wave of 256x256 CTA-pair tiles is split into halves."""
    m, n, k = shape
    a, b = _operands(m, n, k, seed=21)
    aq, sa = _q(ops, a)
    bq, sb = _q(ops, b)
    acc = ops.gemm(aq, bq, "int8", output_dtype=torch.int32).cpu()
    expect = co.gemm_i8_acc_fast(aq.cpu(), bq.cpu())
    assert torch.equal(acc, expect)
    y = ops.gemm(aq, bq, "int8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16).cpu()
    assert torch.equal(y, co.gemm_epilogue(expect, sa.cpu(), sb.cpu()))


@pytest.mark.parametrize("mode", ["int8", "fp8"])
@pytest.mark.parametrize("block", [0, 128])
def test_linear_one_call_equals_two_calls(ops, mode, block):
    m, n, k = 300, 520, 1024
    a, b = _operands(m, n, k, seed=31)
    signs = torch.from_numpy(ref.hadamard_signs(k, 9)).to(DEV) if block else None
    if block:
        wq, ws = ops.hadamard_quantize(b.to(DEV), block, signs, mode)
        aq, sa = ops.hadamard_quantize(a.to(DEV), block, signs, mode)
    else:
        wq, ws = _q(ops, b, mode)
        aq, sa = _q(ops, a, mode)
    two = ops.gemm(aq, wq, mode, a_scales=sa, b_scales=ws, output_dtype=torch.bfloat16)
    one = ops.linear(a.to(DEV), wq, ws, mode, block_size=block, signs=signs)
    one_again = ops.linear(a.to(DEV), wq, ws, mode, block_size=block, signs=signs)
    assert torch.equal(one, two) and torch.equal(one_again, two)


def test_linear_rejects_bad_k(ops):
    x = torch.ones(4, 40, device=DEV, dtype=torch.bfloat16)
    wq = torch.ones(8, 40, device=DEV, dtype=torch.int8)
    with pytest.raises(NotImplementedError, match="16"):
        ops.linear(x, wq, torch.ones(8, device=DEV))


FP32_SHAPES = [(1, 33, 5), (127, 65, 96), (300, 520, 1023), (512, 2048, 2048), (1000, 1000, 3000),
               (64, 96, 16384)]


@pytest.mark.parametrize("shape", FP32_SHAPES)
def test_fp32_gemm_has_fp32_accuracy(ops, shape):
    """FP32 operands (reference mode "fp32", src/m5kernels/metal.py:158-269): three
    TF32 tensor-core products of the operands' TF32 parts, over K chunks of <= 2048
    whose fp32 results are added.  Bar: relative L2 <= 5e-5 against the float64
    product at every K (the reference accepts 1e-4, src/m5kernels/engine.py:473),
    every output within 1e-4 of its |A| |B| scale; bf16 output is the fp32
    result rounded; any K (the parts are zero-padded internally)."""
    m, n, k = shape
    g = torch.Generator().manual_seed(53)
    a = torch.randn(m, k, generator=g) * 3.0
    b = torch.randn(n, k, generator=g) * 0.02
    y = ops.gemm(a.to(DEV), b.to(DEV), "fp32").cpu()
    assert y.dtype == torch.float32
    ref64 = a.double() @ b.double().T
    assert ref.metrics(y.double().numpy(), ref64.numpy())["relative_l2"] <= 5e-5
    scale = (a.double().abs() @ b.double().abs().T)
    assert float(((y.double() - ref64).abs() / scale.clamp_min(1e-30)).max()) <= 1e-4
    yb = ops.gemm(a.to(DEV), b.to(DEV), "fp32", output_dtype=torch.bfloat16).cpu()
    assert torch.equal(yb, y.to(torch.bfloat16))


def test_fp32_gemm_special_values_and_contract(ops):
    """Infinities and NaNs propagate; scales, bias and gate are refused as for the
    other float modes; the C entry point without a workspace says what it needs."""
    from m5kernels_b200 import _lib

    a = torch.ones(4, 8)
    b = torch.ones(3, 8)
    a[1, 2] = float("inf")
    a[2, 0] = float("nan")
    y = ops.gemm(a.to(DEV), b.to(DEV), "fp32").cpu()
    assert torch.isinf(y[1]).all() and torch.isnan(y[2]).all()
    assert torch.equal(y[0], torch.full((3,), 8.0)) and torch.equal(y[3], torch.full((3,), 8.0))
    with pytest.raises(ValueError):
        ops.gemm(a.to(DEV), b.to(DEV), "fp32", a_scales=torch.ones(4, device=DEV),
                 b_scales=torch.ones(3, device=DEV))
    with pytest.raises(NotImplementedError, match="INT8 only"):
        ops.gemm(a.to(DEV), b.to(DEV), "fp32", bias=torch.ones(3, device=DEV))
    out = torch.empty(4, 3, device=DEV)
    ad, bd = a.to(DEV), b.to(DEV)
    rc = _lib.lib().m5b_gemm(ad.data_ptr(), bd.data_ptr(), 4, 3, 8, _lib.MODE["fp32"], None, None,
                             out.data_ptr(), _lib.F32, None, None, 0, None, None, None, 0, None)
    assert rc == _lib.EINVAL and b"workspace" in _lib.lib().m5b_last_error()
