"""GPU parity of the staged comparators (unfused_norm, gated_residual_add, qk_norm_rope).

The reference keeps these stages as standalone kernels so that each fused
kernel can be compared with the same arithmetic split over launches
(src/m5kernels/norm_hadamard.py:280-348, qk_rope.py:185-203).  Bars:
  * each stage bit-exact against the C restatement (oracle/m5_oracle.c);
  * staged pipeline == fused kernel, bit for bit (the reference requires this
    for INT8 Q/K, tests/test_qk_rope_metal.py:78-81, and for the gated update,
    tests/test_gated_norm_hadamard_metal.py:58-61);
  * within the reference's own tolerances of its float64 references
    (tests/test_norm_hadamard_metal.py:150-174: rtol 2e-6 fp32, 1e-3 fp16,
    8e-3 bf16; tests/test_gated_norm_hadamard_metal.py:53-56).
"""

import numpy as np
import pytest
import torch

from oracle import c_oracle as co
from oracle import reference_numpy as ref

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {torch.float32: 2e-6, torch.float16: 1e-3, torch.bfloat16: 8e-3}


@pytest.fixture(scope="module")
def ops():
    import m5kernels_b200 as m

    return m


def _x(rows, k, dtype, seed=0, kind="normal"):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g)
    if kind == "outliers":
        x[:, ::31] *= 30
    elif kind == "zeros":
        x.zero_()
    return x.to(dtype)


def _mod(k, dtype=torch.float32, table=None, seed=3):
    g = torch.Generator().manual_seed(seed)
    gamma = torch.empty(k).uniform_(0.5, 1.5, generator=g).to(dtype)
    shape = (table, k) if table else (k,)
    scale = torch.empty(shape).uniform_(-0.3, 0.3, generator=g).to(dtype)
    shift = torch.empty(shape).uniform_(-0.1, 0.1, generator=g).to(dtype)
    return gamma, scale, shift


# ---------------------------------------------------------------- unfused_norm
@pytest.mark.parametrize("norm", ["rms", "layer"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("round_output", ["input", "fp32"])
@pytest.mark.parametrize("shape", [(3, 5376), (5, 4096), (3, 200), (2, 16384), (300, 1024)])
def test_unfused_norm_oracle_and_reference(ops, norm, dtype, round_output, shape):
    rows, k = shape
    x = _x(rows, k, dtype, seed=79, kind="outliers" if rows == 5 else "normal")
    gamma, scale, shift = _mod(k)
    y = ops.unfused_norm(x.to(DEV), gamma.to(DEV), scale.to(DEV), shift.to(DEV), norm=norm,
                         round_output=round_output)
    out_dtype = dtype if round_output == "input" else torch.float32
    assert y.dtype == out_dtype and tuple(y.shape) == (rows, k)
    o = co.row_prep(x, norm=norm, eps=1e-5, round_output=round_output == "input", gamma=gamma,
                    scale=scale, shift=shift, out="f32")["y"]
    assert torch.equal(y.cpu().float(), o), "differs from the C restatement"
    r = ref.norm_modulate_reference(x.float().numpy(), gamma.numpy(), scale.numpy(),
                                    shift.numpy(), norm=norm)
    r = torch.from_numpy(r.astype(np.float32)).to(out_dtype).float().numpy()
    out = y.cpu().float().numpy()
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, r, rtol=TOL[out_dtype], atol=2e-7)


@pytest.mark.parametrize("norm", ["rms", "layer"])
@pytest.mark.parametrize("dtype,round_output", [(torch.bfloat16, "input"), (torch.float16, "input"),
                                                (torch.bfloat16, "fp32"), (torch.float32, "input")])
@pytest.mark.parametrize("block", [128, 256])
def test_unfused_norm_then_rotation_equals_fused(ops, norm, dtype, round_output, block):
    """unfused_norm -> hadamard_quantize reproduces fused_norm_hadamard_quantize exactly."""
    rows, k = 64, 4096
    x = _x(rows, k, dtype, seed=5)
    gamma, scale, shift = _mod(k, dtype, table=2)
    row_map = (torch.arange(rows, dtype=torch.int32) * 7) % 2
    signs = torch.from_numpy(ref.hadamard_signs(k, 11)).to(DEV)
    args = (x.to(DEV), gamma.to(DEV), scale.to(DEV), shift.to(DEV))
    y = ops.unfused_norm(*args, norm=norm, round_output=round_output, row_map=row_map.to(DEV),
                         epsilon=1e-6)
    sq, ss = ops.hadamard_quantize(y, block, signs, "int8")
    fq, fs = ops.fused_norm_hadamard_quantize(*args, signs, block, norm=norm,
                                              round_output=round_output, row_map=row_map.to(DEV),
                                              epsilon=1e-6)
    assert torch.equal(sq, fq) and torch.equal(ss, fs)


@pytest.mark.parametrize("round_output", ["input", "fp32"])
def test_unfused_norm_explicit_bf16_rounding_ties(ops, round_output):
    """gamma = 0 isolates the post-modulation cast: halfway shifts round to even."""
    width = 256
    shift = torch.tensor([1.00390625, 1.01171875, -1.00390625, -1.01171875]).repeat(width // 4)
    x = torch.zeros(3, width, dtype=torch.bfloat16, device=DEV)
    z = torch.zeros(width, device=DEV)
    y = ops.unfused_norm(x, z, z, shift.to(DEV), round_output=round_output).cpu().float()
    expect = shift.to(torch.bfloat16).float() if round_output == "input" else shift
    assert torch.equal(y, expect.expand(3, width))


@pytest.mark.parametrize("norm", ["rms", "layer"])
def test_unfused_norm_row_map_equals_direct(ops, norm):
    x = _x(7, 768, torch.bfloat16, seed=61).to(DEV)
    gamma, scale, shift = (t.to(DEV) for t in _mod(768, table=3, seed=61))
    row_map = torch.tensor([2, 0, 1, 0, 2, 2, 1], dtype=torch.int32, device=DEV)
    mapped = ops.unfused_norm(x, gamma, scale, shift, norm=norm, row_map=row_map)
    for row, index in enumerate(row_map.tolist()):
        direct = ops.unfused_norm(x[row:row + 1], gamma, scale[index], shift[index], norm=norm)
        assert torch.equal(mapped[row], direct[0])


def test_unfused_norm_layer_constant_rows(ops):
    """LayerNorm of a constant row is exactly zero, leaving the shift."""
    x = torch.full((7, 5376), 17.0, device=DEV)
    gamma = torch.ones(5376, device=DEV)
    scale = torch.full((5376,), 0.5, device=DEV)
    shift = torch.linspace(-1, 1, 5376, device=DEV)
    y = ops.unfused_norm(x, gamma, scale, shift, norm="layer", round_output="fp32")
    assert torch.equal(y, shift.expand(7, 5376))


# ---------------------------------------------------------------- gated_residual_add
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("mapped", [False, True])
@pytest.mark.parametrize("shape", [(64, 4096), (3, 769), (5, 5376), (300, 1024)])
def test_gated_residual_add_oracle_and_reference(ops, dtype, mapped, shape):
    rows, k = shape
    g = torch.Generator().manual_seed(47)
    res = torch.randn(rows, k, generator=g).to(dtype)
    br = torch.randn(rows, k, generator=g).to(dtype)
    gate = (0.1 * torch.randn(3, k, generator=g)).to(torch.bfloat16)
    grm = (torch.arange(rows, dtype=torch.int32) * 5) % 3 if mapped else None
    gate = gate if mapped else gate[1]
    out = ops.gated_residual_add(res.to(DEV), br.to(DEV), gate.to(DEV),
                                 gate_row_map=grm.to(DEV) if mapped else None).cpu()
    assert out.dtype == dtype and out.shape == res.shape
    o = co.row_prep(res, branch=br, gate=gate, gate_row_map=grm, out="f32")["residual"]
    assert torch.equal(out, o), "differs from the C restatement"
    ideal = ref.gated_residual_reference(res.float().numpy(), br.float().numpy(),
                                         gate.float().numpy(),
                                         row_map=grm.numpy() if mapped else None)
    expect = torch.from_numpy(ideal.astype(np.float32)).to(dtype).float().numpy()
    np.testing.assert_allclose(out.float().numpy(), expect,
                               rtol={torch.bfloat16: 8e-3, torch.float16: 1e-3,
                                     torch.float32: 3e-7}[dtype], atol=1e-7)


@pytest.mark.parametrize("mapped", [False, True])
@pytest.mark.parametrize("norm", ["rms", "layer"])
def test_gated_add_then_fused_norm_equals_fused_gated(ops, mapped, norm):
    """The fair two-launch baseline reproduces the one-kernel gated path exactly."""
    rows, k = 256, 4096
    g = torch.Generator().manual_seed(17)
    res = torch.randn(rows, k, generator=g).to(torch.bfloat16).to(DEV)
    br = torch.randn(rows, k, generator=g).to(torch.bfloat16).to(DEV)
    gate = (0.1 * torch.randn(2, k, generator=g)).to(torch.bfloat16).to(DEV)
    gate = gate if mapped else gate[0].contiguous()
    grm = (torch.arange(rows, dtype=torch.int32, device=DEV) // 128) if mapped else None
    gamma, scale, shift = (t.to(DEV) for t in _mod(k, torch.bfloat16, table=2))
    rm = torch.arange(rows, dtype=torch.int32, device=DEV) % 2
    signs = torch.from_numpy(ref.hadamard_signs(k, 23)).to(DEV)
    fq, fs, fr = ops.fused_gated_residual_norm_hadamard_quantize(
        res, br, gate, gamma, scale, shift, signs, 128, norm=norm, epsilon=1e-6,
        gate_row_map=grm, row_map=rm)
    staged_r = ops.gated_residual_add(res, br, gate, gate_row_map=grm)
    sq, ss = ops.fused_norm_hadamard_quantize(staged_r, gamma, scale, shift, signs, 128,
                                              norm=norm, epsilon=1e-6, row_map=rm)
    assert torch.equal(staged_r, fr)
    assert torch.equal(sq, fq) and torch.equal(ss, fs)


def test_gated_residual_add_exact_cancellation_and_strided(ops):
    """R = -branch * gate exactly cancels (no early product rounding); strided inputs."""
    k = 769
    g = torch.Generator().manual_seed(313)
    branch = torch.randn(k, 3, generator=g).to(torch.bfloat16).T  # strided [3, 769]
    gate = torch.full((k,), -0.5)
    residual = (branch.float() * 0.5).to(torch.bfloat16)  # exact: halving a bf16
    out = ops.gated_residual_add(residual.to(DEV), branch.to(DEV), gate.to(DEV)).cpu()
    assert torch.equal(out, torch.zeros(3, k, dtype=torch.bfloat16))
    # (1 + 2^-7)^2 = 1 + 2^-6 + 2^-14 is not a bf16; kept in FP32 until the add,
    # R = -(1 + 2^-6) leaves 2^-14 (a bf16 product would leave 0)
    r = torch.full((1, 8), -(1.0 + 2.0**-6), dtype=torch.bfloat16)
    b = torch.full((1, 8), 1.0 + 2.0**-7, dtype=torch.bfloat16)
    gt = torch.full((8,), 1.0 + 2.0**-7, dtype=torch.bfloat16)
    out = ops.gated_residual_add(r.to(DEV), b.to(DEV), gt.to(DEV)).cpu()
    assert torch.equal(out, torch.full((1, 8), 2.0**-14, dtype=torch.bfloat16))


def test_gate_contract_rejections(ops):
    residual = torch.zeros(3, 768, device=DEV)
    branch = torch.zeros(3, 768, device=DEV)
    gate = torch.ones(768, device=DEV)
    with pytest.raises(ValueError, match="branch"):
        ops.gated_residual_add(residual, torch.zeros(2, 768, device=DEV), gate)
    with pytest.raises(ValueError, match="floating dtype"):
        ops.gated_residual_add(residual, branch, gate.to(torch.int8))
    with pytest.raises(ValueError, match="vector of length K"):
        ops.gated_residual_add(residual, branch, torch.ones(2, 768, device=DEV))
    with pytest.raises(ValueError, match="int32 vector"):
        ops.gated_residual_add(residual, branch, torch.ones(2, 768, device=DEV),
                               gate_row_map=torch.zeros(3, device=DEV))
    with pytest.raises(NotImplementedError, match="threadgroup sizes"):
        ops.gated_residual_add(residual, branch, gate, threads=64)


# ---------------------------------------------------------------- qk_norm_rope
def _qk_tables(m, half, seed):
    g = torch.Generator().manual_seed(seed)
    gamma = (1 + 0.02 * torch.randn(128, generator=g)).to(torch.bfloat16)
    ang = (torch.rand(m, half, generator=g) * 2 - 1) * np.pi
    return gamma, torch.cos(ang).to(torch.bfloat16), torch.sin(ang).to(torch.bfloat16)


@pytest.mark.parametrize("shape,half", [((5, 384), 1), ((5, 384), 48), ((5, 384), 64),
                                        ((300, 512), 33), ((4096, 1024), 64), ((33, 128), 8)])
def test_qk_norm_rope_oracle_and_reference(ops, shape, half):
    m, n = shape
    g = torch.Generator().manual_seed(713)
    p = torch.randn(m, n // 128, 128, generator=g)
    p[0] = 0
    if m > 1:
        p[1, :, ::31] *= 100
    p = p.reshape(m, n).to(torch.bfloat16)
    gamma, cos, sin = _qk_tables(m, half, 713)
    y = ops.qk_norm_rope(p.to(DEV), gamma.to(DEV), cos.to(DEV), sin.to(DEV)).cpu()
    assert tuple(y.shape) == (n // 128, m, 128)
    expect = co.qk_rope_from_acc(p.float(), None, None, gamma, cos, sin, half, 1e-5)
    assert torch.equal(y, expect)
    assert torch.equal(y[:, 0], torch.zeros(n // 128, 128, dtype=torch.bfloat16))
    r = ref.qk_rope_reference(p.float().numpy().reshape(m, n // 128, 128), gamma.float().numpy(),
                              cos.float().numpy(), sin.float().numpy())["output"]
    yd = y.double().numpy()
    ulp = np.abs(yd - r) / np.maximum(np.abs(r) * 2.0**-7, 2.0**-133)
    assert ulp.max() <= 2 or ref.metrics(yd, r)["relative_l2"] <= 1e-3


@pytest.mark.parametrize("shape,half", [((300, 512, 1024), 64), ((512, 384, 256), 48),
                                        ((129, 256, 192), 64), ((1000, 1024, 512), 37)])
def test_staged_projection_then_norm_equals_fused(ops, shape, half):
    """gemm(int8 -> bf16) -> qk_norm_rope == projection_qk_rope, bit for bit."""
    m, n, k = shape
    g = torch.Generator().manual_seed(29)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV)
    w = (torch.randn(n, k, generator=g) * k ** -0.5).to(torch.bfloat16).to(DEV)
    gamma, cos, sin = (t.to(DEV) for t in _qk_tables(m, half, 29))
    aq, sa = ops.quantize(x, "int8")
    bq, sb = ops.quantize(w, "int8")
    fused = ops.projection_qk_rope(aq, bq, gamma, cos, sin, "int8", a_scales=sa, b_scales=sb)
    proj = ops.gemm(aq, bq, "int8", a_scales=sa, b_scales=sb, output_dtype=torch.bfloat16)
    staged = ops.qk_norm_rope(proj, gamma, cos, sin)
    assert torch.equal(fused, staged)


def test_qk_norm_rope_pairing_and_head_major(ops):
    p = torch.ones(3, 2, 128)
    p[:, :, 48:96] = -1
    p[:, 1] *= -1
    pb = p.reshape(3, 256).to(torch.bfloat16)
    gamma = torch.ones(128, dtype=torch.bfloat16)
    cos = torch.zeros(3, 48, dtype=torch.bfloat16)
    sin = torch.ones(3, 48, dtype=torch.bfloat16)
    y = ops.qk_norm_rope(pb.to(DEV), gamma.to(DEV), cos.to(DEV), sin.to(DEV)).cpu().float()
    expect = p.clone()
    expect[:, :, :48] = -p[:, :, 48:96]
    expect[:, :, 48:96] = p[:, :, :48]
    assert torch.equal(y, expect.transpose(0, 1))


def test_qk_norm_rope_contract(ops):
    p = torch.zeros(4, 256, dtype=torch.bfloat16, device=DEV)
    gamma = torch.ones(128, dtype=torch.bfloat16, device=DEV)
    cos = torch.ones(4, 64, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError, match="bfloat16"):
        ops.qk_norm_rope(p.float(), gamma, cos, cos)
    with pytest.raises(ValueError, match="128-wide heads"):
        ops.qk_norm_rope(p[:, :200], gamma, cos, cos)
    with pytest.raises(NotImplementedError, match="128 or 256 threads"):
        ops.qk_norm_rope(p, gamma, cos, cos, threads=64)
    with pytest.raises(ValueError, match="epsilon"):
        ops.qk_norm_rope(p, gamma, cos, cos, epsilon=0.0)
