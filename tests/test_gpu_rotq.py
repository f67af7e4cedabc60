"""Parity of the lean rotate(+quantize) kernel for plain rows.

Rows without normalization or gate, rotated with B >= 64 and K / 64 a power
of two below 32 or a multiple of 32 up to 256, run on the row-group kernel
(several rows per CTA step, packed FP32 butterflies).  Its codes, scales and
rotated values must equal the C restatement bit for bit, for every input
dtype, output kind and row-group shape, including a partial last row group,
rows with half-integer quotients, and zero rows.
"""

import numpy as np
import pytest
import torch

from oracle import c_oracle as co
from oracle import reference_numpy as ref

pytestmark = pytest.mark.gpu

DEV = "cuda"

# (rows, K, block): threads per row K/64 = 4, 8, 16, 32, 64, 96, 128, 256
SHAPES = [(1000, 256, 64), (777, 512, 128), (513, 1024, 256), (300, 2048, 1024),
          (259, 4096, 256), (130, 6144, 128), (65, 8192, 512), (33, 16384, 128)]


def _rows(m, k, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g)
    cols = torch.randperm(k, generator=g)[: max(1, k // 100)]
    x[:, cols] *= 30
    x[m // 3] = 0.0
    # a few rows whose rotated values sit on half-integer quotients are not
    # constructible directly; exact ties come from small-integer rows instead
    x[m // 2] = torch.randint(-3, 4, (k,), generator=g).float()
    return x.to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", SHAPES, ids=[f"{m}x{k}b{b}" for m, k, b in SHAPES])
@pytest.mark.parametrize("out", ["int8", "fp8", "f32"])
def test_lean_rotate_quantize_bit_exact(dtype, shape, out):
    import m5kernels_b200 as m5

    m, k, block = shape
    x = _rows(m, k, dtype, seed=k + block)
    signs = torch.from_numpy(ref.hadamard_signs(k, 3))
    if out == "f32":
        y = m5.rotate(x.to(DEV), block, signs.to(DEV)).cpu()
        assert torch.equal(y, co.rotate(x, block, signs))
    else:
        q, s = m5.hadamard_quantize(x.to(DEV), block, signs.to(DEV), out)
        o = co.row_prep(x, block=block, signs=signs, out=out)
        assert torch.equal(s.cpu(), o["s"])
        assert torch.equal(q.cpu(), o["q"])


def test_lean_matches_float64_reference():
    import m5kernels_b200 as m5

    m, k, block = 259, 4096, 256
    x = _rows(m, k, torch.bfloat16, seed=1)
    signs = torch.from_numpy(ref.hadamard_signs(k, 9))
    y = m5.rotate(x.to(DEV), block, signs.to(DEV)).cpu().numpy()
    y64 = ref.block_hadamard_reference(x.float().numpy(), block, signs.numpy())
    assert ref.metrics(y, y64)["relative_l2"] <= 1e-6
    q, s = m5.hadamard_quantize(x.to(DEV), block, signs.to(DEV), "int8")
    rq, rs = ref.quantize_reference(y64.astype(np.float32), "int8")
    assert np.abs(q.cpu().numpy().astype(np.int16) - rq.astype(np.int16)).max() <= 1


# Normalized rows on the lean kernel: (rows, K, block) over the unit shapes,
# blocks 64..256, RMS and LayerNorm, with and without the gated residual,
# per-row modulation tables, INT8 and E4M3, bf16 / f16 / f32 inputs.
NORM_SHAPES = [(300, 512, 64), (129, 2048, 128), (97, 4096, 256), (33, 6144, 128),
               (17, 16384, 64)]


def _tables(k, p, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    gamma = (1 + 0.1 * torch.randn(k, generator=g)).to(dtype)
    scale = (0.2 * torch.randn(p, k, generator=g)).to(dtype)
    shift = (0.1 * torch.randn(p, k, generator=g)).to(dtype)
    gate = (0.3 * torch.randn(p, k, generator=g)).to(dtype)
    return gamma, scale, shift, gate


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", NORM_SHAPES, ids=[f"{m}x{k}b{b}" for m, k, b in NORM_SHAPES])
@pytest.mark.parametrize("norm", ["rms", "layer"])
@pytest.mark.parametrize("gated", [False, True])
def test_lean_norm_bit_exact(dtype, shape, norm, gated):
    import m5kernels_b200 as m5

    m, k, block = shape
    x = _rows(m, k, dtype, seed=k + 7)
    p = 3
    gamma, scale, shift, gate = _tables(k, p, dtype, seed=k)
    rm = (torch.arange(m, dtype=torch.int32) * 5) % p
    grm = (torch.arange(m, dtype=torch.int32) * 7 + 1) % p
    signs = torch.from_numpy(ref.hadamard_signs(k, 5))
    out = "fp8" if (k == 2048 and dtype != torch.float32) else "int8"
    common = dict(norm=norm, epsilon=1e-6, row_map=rm.to(DEV), out=out)
    if gated:
        br = _rows(m, k, dtype, seed=k + 11)
        q, s, r2 = m5.fused_gated_residual_norm_hadamard_quantize(
            x.to(DEV), br.to(DEV), gate.to(DEV), gamma.to(DEV), scale.to(DEV), shift.to(DEV),
            signs.to(DEV), block, gate_row_map=grm.to(DEV), **common)
        o = co.row_prep(x, block=block, norm=norm, eps=1e-6, round_output=True, gamma=gamma,
                        scale=scale, shift=shift, row_map=rm, signs=signs, branch=br, gate=gate,
                        gate_row_map=grm, out=out)
        assert torch.equal(r2.cpu(), o["residual"])
    else:
        q, s = m5.fused_norm_hadamard_quantize(
            x.to(DEV), gamma.to(DEV), scale.to(DEV), shift.to(DEV), signs.to(DEV), block, **common)
        o = co.row_prep(x, block=block, norm=norm, eps=1e-6, round_output=True, gamma=gamma,
                        scale=scale, shift=shift, row_map=rm, signs=signs, out=out)
    assert torch.equal(s.cpu(), o["s"])
    assert torch.equal(q.cpu(), o["q"])
