"""GPU parity of the row-preparation kernels (quantize / rotate / fused prep).

Bar: codes and scales bit-exact against the C restatement (same FP32
reduction order); plain quantization bit-exact against the reference's own
quantize_reference; fused prep within the reference's own GPU tolerance
(<= 1 code, scales rtol 3e-5; tests/test_norm_hadamard_metal.py:75-76 in the
reference) against the float64 ideal; the updated residual exactly equal to
the float64 update rounded FP32 -> BF16 (norm_hadamard_gemm.py:121-132).
"""

import numpy as np
import pytest
import torch

from oracle import c_oracle as co
from oracle import reference_numpy as ref

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _x(rows, k, dtype, kind="normal", seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g)
    if kind == "zeros":
        x.zero_()
    elif kind == "outliers":
        x[:, ::31] *= 30
    elif kind == "rowzero":
        x[rows // 2] = 0
    return x.to(dtype)


@pytest.fixture(scope="module")
def ops():
    import m5kernels_b200 as m

    return m


@pytest.mark.parametrize("mode", ["int8", "fp8"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("kind", ["normal", "zeros", "outliers", "rowzero"])
# K = 2048 * 2^k (16-bit) and 1024 * 2^k (fp32) run the exact-fit quantize instances (every
# thread's vectors in bounds, no guards); the others keep the per-vector bounds checks.
@pytest.mark.parametrize("shape", [(7, 256), (3, 257), (1, 33), (9, 5376), (4, 16384), (5, 5384),
                                   (3, 200), (2, 32768), (300, 1024), (6, 2048), (3, 4096),
                                   (5, 8192)])
def test_quantize_matches_reference_bit_exact(ops, mode, dtype, kind, shape):
    x = _x(*shape, dtype, kind)
    q, s = ops.quantize(x.to(DEV), mode)
    rq, rs = ref.quantize_reference(x.float().numpy(), mode)
    np.testing.assert_array_equal(q.cpu().numpy().view(np.uint8), rq.view(np.uint8))
    np.testing.assert_array_equal(s.cpu().numpy(), rs.astype(np.float32))


def test_quantize_golden(ops, golden):
    xb = torch.from_numpy(golden["quant_x_bf16"].view(np.int16)).view(torch.bfloat16)
    for mode in ("int8", "fp8"):
        q, s = ops.quantize(xb.to(DEV), mode)
        np.testing.assert_array_equal(q.cpu().numpy().view(np.uint8),
                                      golden[f"quant_{mode}_q"].view(np.uint8))
        np.testing.assert_array_equal(s.cpu().numpy(), golden[f"quant_{mode}_s"])
    x32 = torch.from_numpy(golden["quant_x_f32_oddk"])
    q, s = ops.quantize(x32.to(DEV), "int8")
    np.testing.assert_array_equal(q.cpu().numpy(), golden["quant_oddk_int8_q"])
    np.testing.assert_array_equal(s.cpu().numpy(), golden["quant_oddk_int8_s"])


@pytest.mark.parametrize("block", [32, 64, 128, 256, 512, 1024])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rotate_bit_exact_vs_oracle_and_close_to_float64(ops, block, dtype):
    k = block * 3
    x = _x(5, k, dtype, seed=block)
    signs = torch.from_numpy(ref.hadamard_signs(k, 17))
    y = ops.rotate(x.to(DEV), block, signs.to(DEV)).cpu()
    yo = co.rotate(x, block, signs)
    assert torch.equal(y, yo)
    y64 = ref.block_hadamard_reference(x.float().numpy(), block, signs.numpy())
    assert ref.metrics(y.numpy(), y64)["relative_l2"] <= 1e-6


def test_rotate_golden(ops, golden):
    x = torch.from_numpy(golden["rot_x"])
    signs = torch.from_numpy(golden["signs_k512_seed17"])
    for b in (32, 128, 256, 512):
        y = ops.rotate(x.to(DEV), b, signs.to(DEV)).cpu().numpy()
        assert ref.metrics(y, golden[f"rot_b{b}"])["relative_l2"] <= 1e-6


@pytest.mark.parametrize("mode", ["int8", "fp8"])
@pytest.mark.parametrize("block", [128, 256])
def test_hadamard_quantize_equals_two_step(ops, mode, block):
    k = 4096
    x = _x(33, k, torch.bfloat16, "outliers")
    signs = torch.from_numpy(ref.hadamard_signs(k, 5)).to(DEV)
    q, s = ops.hadamard_quantize(x.to(DEV), block, signs, mode)
    q2, s2 = ops.quantize(ops.rotate(x.to(DEV), block, signs), mode)
    assert torch.equal(q, q2) and torch.equal(s, s2)
    o = co.row_prep(x, block=block, signs=signs.cpu(), out=mode)
    assert torch.equal(q.cpu(), o["q"]) and torch.equal(s.cpu(), o["s"])


def _mod_params(k, dtype=torch.float32, table=None, seed=3):
    g = torch.Generator().manual_seed(seed)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(dtype)
    shape = (table, k) if table else (k,)
    scale = (0.2 * torch.randn(*shape, generator=g)).to(dtype)
    shift = (0.1 * torch.randn(*shape, generator=g)).to(dtype)
    return gamma, scale, shift


def _check_vs_float64(q, s, x, gamma, scale, shift, signs, block, norm, eps, round_dtype,
                      row_map=None):
    xf = x.float().numpy()
    if row_map is None:
        mod = ref.norm_modulate_reference(xf, gamma.float().numpy(), scale.float().numpy(),
                                          shift.float().numpy(), norm=norm, eps=eps)
    else:
        rm = row_map.numpy()
        mod = np.concatenate([
            ref.norm_modulate_reference(xf[i:i + 1], gamma.float().numpy(), scale[rm[i]].float().numpy(),
                                        shift[rm[i]].float().numpy(), norm=norm, eps=eps)
            for i in range(xf.shape[0])])
    if round_dtype is not None:
        mod = torch.from_numpy(mod.astype(np.float32)).to(round_dtype).float().numpy()
    rot = ref.block_hadamard_reference(mod, block, signs.numpy())
    rq, rs = ref.quantize_reference(rot, "int8")
    diff = np.abs(q.numpy().astype(np.int16) - rq.astype(np.int16))
    assert diff.max() <= 1
    np.testing.assert_allclose(s.numpy(), rs, rtol=3e-5, atol=1e-7)


@pytest.mark.parametrize("norm", ["rms", "layer"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("kind", ["normal", "zeros", "outliers"])
@pytest.mark.parametrize("round_output", ["input", "fp32"])
def test_fused_prep_h3_width(ops, norm, dtype, kind, round_output):
    k = 5376
    x = _x(7, k, dtype, kind, seed=621)
    gamma, scale, shift = _mod_params(k)
    signs = torch.from_numpy(ref.hadamard_signs(k, 29))
    q, s = ops.fused_norm_hadamard_quantize(
        x.to(DEV), gamma.to(DEV), scale.to(DEV), shift.to(DEV), signs.to(DEV), 256, norm=norm,
        round_output=round_output)
    q, s = q.cpu(), s.cpu()
    o = co.row_prep(x, block=256, norm=norm, eps=1e-5, round_output=round_output == "input",
                    gamma=gamma, scale=scale, shift=shift, signs=signs)
    assert torch.equal(q, o["q"]), "codes differ from the C restatement"
    assert torch.equal(s, o["s"]), "scales differ from the C restatement"
    _check_vs_float64(q, s, x, gamma, scale, shift, signs, 256, norm, 1e-5,
                      dtype if (round_output == "input" and dtype != torch.float32) else None)


@pytest.mark.parametrize("block", [32, 64, 128, 256, 512, 1024])
@pytest.mark.parametrize("norm", ["rms", "layer"])
def test_fused_prep_blocks_and_partial_warps(ops, block, norm):
    k = block * 3
    x = _x(3, k, torch.float32, seed=31)
    gamma = torch.ones(k)
    scale = torch.full((k,), 0.125)
    shift = torch.full((k,), 0.0625)
    signs = torch.from_numpy(ref.hadamard_signs(k, 13))
    q, s = ops.fused_norm_hadamard_quantize(x.to(DEV), gamma.to(DEV), scale.to(DEV),
                                            shift.to(DEV), signs.to(DEV), block, norm=norm,
                                            threads=128)
    o = co.row_prep(x, block=block, norm=norm, eps=1e-5, round_output=True, gamma=gamma,
                    scale=scale, shift=shift, signs=signs)
    assert torch.equal(q.cpu(), o["q"]) and torch.equal(s.cpu(), o["s"])
    _check_vs_float64(q.cpu(), s.cpu(), x, gamma, scale, shift, signs, block, norm, 1e-5, None)


@pytest.mark.parametrize("mode", ["int8", "fp8"])
def test_fused_prep_row_map_and_fp8(ops, mode):
    m, k = 4096, 4096
    x = _x(m, k, torch.bfloat16, seed=9)
    gamma, scale, shift = _mod_params(k, torch.bfloat16, table=2)
    row_map = (torch.arange(m, dtype=torch.int32) // 2048)
    signs = torch.ones(k, dtype=torch.int8)
    q, s = ops.fused_norm_hadamard_quantize(
        x.to(DEV), gamma.to(DEV), scale.to(DEV), shift.to(DEV), signs.to(DEV), 128, norm="layer",
        epsilon=1e-6, row_map=row_map.to(DEV), out=mode)
    o = co.row_prep(x, block=128, norm="layer", eps=1e-6, round_output=True, gamma=gamma,
                    scale=scale, shift=shift, row_map=row_map, signs=signs, out=mode)
    assert torch.equal(q.cpu(), o["q"]) and torch.equal(s.cpu(), o["s"])


@pytest.mark.parametrize("mapped", [False, True])
@pytest.mark.parametrize("norm", ["rms", "layer"])
def test_gated_residual_prep(ops, mapped, norm):
    m, k = 64, 4096
    g = torch.Generator().manual_seed(47)
    res = torch.randn(m, k, generator=g).to(torch.bfloat16)
    br = torch.randn(m, k, generator=g).to(torch.bfloat16)
    gate = (0.1 * torch.randn(2 if mapped else 1, k, generator=g)).to(torch.bfloat16)
    gate = gate if mapped else gate[0]
    grm = (torch.arange(m, dtype=torch.int32) * 3 % 2) if mapped else None
    gamma, scale, shift = _mod_params(k, torch.bfloat16, table=2)
    rm = torch.arange(m, dtype=torch.int32) // 32
    signs = torch.ones(k, dtype=torch.int8)
    q, s, r2 = ops.fused_gated_residual_norm_hadamard_quantize(
        res.to(DEV), br.to(DEV), gate.to(DEV), gamma.to(DEV), scale.to(DEV), shift.to(DEV),
        signs.to(DEV), 128, norm=norm, epsilon=1e-6,
        gate_row_map=grm.to(DEV) if mapped else None, row_map=rm.to(DEV))
    ideal = ref.gated_residual_reference(res.float().numpy(), br.float().numpy(),
                                         gate.float().numpy(),
                                         row_map=grm.numpy() if mapped else None)
    expect_r = torch.from_numpy(ideal.astype(np.float32)).to(torch.bfloat16)
    assert torch.equal(r2.cpu(), expect_r), "updated residual is not the rounded exact update"
    o = co.row_prep(res, block=128, norm=norm, eps=1e-6, round_output=True, gamma=gamma,
                    scale=scale, shift=shift, row_map=rm, signs=signs, branch=br, gate=gate,
                    gate_row_map=grm)
    assert torch.equal(r2.cpu(), o["residual"])
    assert torch.equal(q.cpu(), o["q"]) and torch.equal(s.cpu(), o["s"])


def test_inputs_not_mutated(ops):
    x = _x(8, 1024, torch.bfloat16).to(DEV)
    before = x.clone()
    gamma, scale, shift = (t.to(DEV) for t in _mod_params(1024))
    signs = torch.ones(1024, dtype=torch.int8, device=DEV)
    ops.fused_norm_hadamard_quantize(x, gamma, scale, shift, signs, 256)
    ops.quantize(x, "int8")
    torch.cuda.synchronize()
    assert torch.equal(x, before)


def test_contract_rejections(ops):
    x = torch.ones(4, 96, device=DEV, dtype=torch.bfloat16)
    signs = torch.ones(96, dtype=torch.int8, device=DEV)
    with pytest.raises(NotImplementedError, match="divisible"):
        ops.rotate(x, 64, signs)
    with pytest.raises(ValueError, match="power of two"):
        ops.rotate(x, 48, signs)
    with pytest.raises(NotImplementedError, match="from 32 through 1024"):
        ops.rotate(torch.ones(2, 16, device=DEV), 16, torch.ones(16, dtype=torch.int8, device=DEV))
    with pytest.raises(ValueError, match="signs"):
        ops.rotate(x, 32, signs.float())


@pytest.mark.parametrize("mode", ["int8", "fp8"])
def test_quantize_misaligned_base(ops, mode):
    rows, k = 6, 4096
    store = torch.randn(rows * k + 16).to(torch.bfloat16)
    x = store[3:3 + rows * k].view(rows, k)  # contiguous, base not 16-byte aligned
    xd = store.to(DEV)[3:3 + rows * k].view(rows, k)
    q, s = ops.quantize(xd, mode)
    rq, rs = ref.quantize_reference(x.float().numpy(), mode)
    np.testing.assert_array_equal(q.cpu().numpy().view(np.uint8), rq.view(np.uint8))
    np.testing.assert_array_equal(s.cpu().numpy(), rs)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("k", [5376, 16384, 32768])
def test_gated_prep_wide_rows_and_padded_ring(ops, dtype, k):
    m = 9
    g = torch.Generator().manual_seed(k)
    res = torch.randn(m, k, generator=g).to(dtype)
    br = torch.randn(m, k, generator=g).to(dtype)
    gate = (0.1 * torch.randn(k, generator=g)).to(torch.bfloat16)
    gamma, scale, shift = _mod_params(k, torch.bfloat16)
    signs = torch.from_numpy(ref.hadamard_signs(k, 3))
    q, s, r2 = ops.fused_gated_residual_norm_hadamard_quantize(
        res.to(DEV), br.to(DEV), gate.to(DEV), gamma.to(DEV), scale.to(DEV), shift.to(DEV),
        signs.to(DEV), 256, norm="rms")
    o = co.row_prep(res, block=256, norm="rms", eps=1e-5, round_output=True, gamma=gamma,
                    scale=scale, shift=shift, signs=signs, branch=br, gate=gate)
    assert torch.equal(r2.cpu(), o["residual"])
    assert torch.equal(q.cpu(), o["q"]) and torch.equal(s.cpu(), o["s"])


@pytest.mark.parametrize("block", [64, 1024])
def test_many_rows_persistent_ring(ops, block):
    """More rows than resident CTAs: every ring slot is reused many times."""
    m, k = 3000, 2048
    x = _x(m, k, torch.bfloat16, "outliers", seed=77)
    signs = torch.from_numpy(ref.hadamard_signs(k, 21))
    gamma, scale, shift = _mod_params(k, torch.bfloat16, table=3)
    rm = (torch.arange(m, dtype=torch.int32) * 7) % 3
    q, s = ops.fused_norm_hadamard_quantize(x.to(DEV), gamma.to(DEV), scale.to(DEV), shift.to(DEV),
                                            signs.to(DEV), block, norm="layer", row_map=rm.to(DEV))
    o = co.row_prep(x, block=block, norm="layer", eps=1e-5, round_output=True, gamma=gamma,
                    scale=scale, shift=shift, row_map=rm, signs=signs)
    assert torch.equal(q.cpu(), o["q"]) and torch.equal(s.cpu(), o["s"])
