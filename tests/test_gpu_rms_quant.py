"""GPU parity of the RMS scale-folding preparation (m5b_rms_quantize).

Bar: codes and scales bit-exact against the C restatement (oracle/m5_oracle.c
m5o_rms_quantize: same FP32 reduction order and operation order), in both the
folded and the direct form, for every input dtype, rotation block and the
ragged / unaligned shapes; against the reference's own float64 vectors
(tests/golden/rms_quant_vectors.npz) within the reference's GPU bound (codes
within one, scales rtol 3e-6; tests/test_rms_quant_metal.py:19-46 of the
reference) and exactly on ties, integer rows and zero rows.
"""

import math

import numpy as np
import pytest
import torch

from oracle import c_oracle as co
from oracle import reference_numpy as ref

pytestmark = pytest.mark.gpu

DEV = "cuda"
DTYPES = [torch.bfloat16, torch.float16, torch.float32]


@pytest.fixture(scope="module")
def ops():
    import m5kernels_b200 as m

    return m


def _signs(k, seed):
    return torch.from_numpy(ref.hadamard_signs(k, seed))


def _inputs(rows, k, dtype, kind, seed=2021):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, k, generator=g)
    gamma = (torch.rand(k, generator=g) * 3.4 - 1.7).float()
    if kind == "zeros":
        x.zero_()
    elif kind == "outliers":
        x[:, ::137] *= 100
    elif kind == "weighted_peak":
        x[:, 0] = 100
        gamma[0] = 1e-3
        gamma[1::31] *= 100
    elif kind == "epsilon":
        x *= 1e-9
    elif kind == "rowzero":
        x[rows // 2] = 0
    return x.to(dtype), gamma


def _run(ops, x, gamma, signs, block, fold, eps=1e-5):
    q, s = ops.rms_quantize(x.to(DEV), gamma.to(DEV), signs.to(DEV), block, fold_scale=fold,
                            epsilon=eps)
    torch.cuda.synchronize()
    return q.cpu(), s.cpu()


def _assert_oracle(ops, x, gamma, signs, block, fold, eps=1e-5):
    q, s = _run(ops, x, gamma, signs, block, fold, eps)
    qo, so = co.rms_quantize(x, gamma, signs, block, fold_scale=fold, epsilon=eps)
    assert torch.equal(q, qo), f"codes differ at {int((q != qo).sum())} places"
    assert torch.equal(s.view(torch.int32), so.view(torch.int32))
    return q, s


SHAPES = [  # rows, K, block
    (7, 5376, 256), (7, 769, 1), (3, 768, 256), (3, 96, 32), (3, 192, 64), (5, 384, 128),
    (3, 1536, 512), (3, 3072, 1024), (64, 4096, 128), (33, 16384, 256), (9, 4096, 1),
    (5, 32768, 1), (4, 32768, 1024), (300, 2048, 64), (2, 24, 1),
]


@pytest.mark.parametrize("fold", [True, False])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,k,block", SHAPES)
def test_bit_exact_against_oracle(ops, rows, k, block, dtype, fold):
    x, gamma = _inputs(rows, k, dtype, "normal", seed=rows * 7 + k)
    _assert_oracle(ops, x, gamma, _signs(k, 61), block, fold)


@pytest.mark.parametrize("fold", [True, False])
@pytest.mark.parametrize("kind", ["zeros", "outliers", "weighted_peak", "epsilon", "rowzero"])
@pytest.mark.parametrize("k,block", [(5376, 256), (769, 1)])
def test_distributions(ops, k, block, kind, fold):
    x, gamma = _inputs(7, k, torch.float32, kind)
    q, s = _assert_oracle(ops, x, gamma, _signs(k, 61), block, fold)
    r = ref.rms_quantize_reference(x.double().numpy(), gamma.double().numpy(),
                                   _signs(k, 61).numpy(), block)
    assert int(np.abs(q.numpy().astype(np.int16) - r["quantized"]).max()) <= 1
    np.testing.assert_allclose(s.numpy(), r["scales"], rtol=3e-6, atol=1e-30)
    if kind == "zeros":
        assert int(q.abs().max()) == 0 and bool((s == 1).all())


GOLDEN = ["h256", "plain769", "outliers", "weighted_peak", "tiny", "eps1", "ties", "zero_row",
          "zero_gamma", "int17", "int257"]
EXACT = {"ties", "zero_row", "zero_gamma", "int17", "int257"}


@pytest.mark.parametrize("fold", [True, False])
@pytest.mark.parametrize("name", GOLDEN)
def test_reference_vectors(ops, rms_golden, name, fold):
    pre = f"rms_{name}_"
    x = torch.from_numpy(rms_golden[pre + "x"])
    gamma = torch.from_numpy(rms_golden[pre + "gamma"])
    signs = torch.from_numpy(rms_golden[pre + "signs"])
    block, eps = int(rms_golden[pre + "block"]), float(rms_golden[pre + "eps"])
    q, s = _assert_oracle(ops, x, gamma, signs, block, fold, eps)
    q_ref, s_ref = rms_golden[pre + "quantized"], rms_golden[pre + "scales"]
    if name in EXACT:
        np.testing.assert_array_equal(q.numpy(), q_ref)
    else:
        assert int(np.abs(q.numpy().astype(np.int16) - q_ref.astype(np.int16)).max()) <= 1
    np.testing.assert_allclose(s.numpy(), s_ref, rtol=3e-6, atol=1e-30)


def test_ties_exact_for_both_forms(ops):
    x = torch.tensor([[127, 2.5, 3.5, -2.5, -3.5, 0, -127, 1.5]], dtype=torch.float32)
    for fold in (True, False):
        q, s = _run(ops, x, torch.ones(8), torch.ones(8, dtype=torch.int8), 1, fold)
        assert q.tolist() == [[127, 2, 4, -2, -4, 0, -127, 2]]
        expected = 1 / math.sqrt(float(np.mean(x.double().numpy() ** 2)) + 1e-5)
        if fold:
            assert math.isclose(float(s[0]), expected, rel_tol=3e-6)


def test_bf16_rows_on_exact_quotients(ops):
    # bf16 rows of half-integers under a peak of 127 with unit gamma put
    # u / peak * 127 exactly on half-integers: the exact fix-up path must agree
    # with the oracle element for element.
    pattern = np.concatenate([[127.0], np.arange(-126, 126) + 0.5]).astype(np.float32)
    x = torch.from_numpy(np.resize(pattern, (64, 4096))).to(torch.bfloat16)
    _assert_oracle(ops, x, torch.ones(4096), torch.ones(4096, dtype=torch.int8), 1, True)
    _assert_oracle(ops, x, torch.ones(4096), _signs(4096, 3), 256, False)


def test_no_bf16_boundary(ops):
    x = torch.ones((3, 256), dtype=torch.bfloat16)
    gamma = torch.ones(256)
    gamma[0] = 1.003
    for fold in (True, False):
        _, s = _run(ops, x, gamma, torch.ones(256, dtype=torch.int8), 1, fold)
        assert bool((torch.abs(s - 1 / 127) > 1e-5).all())


def test_zero_and_signed_gamma(ops):
    x = torch.full((3, 768), 2.0)
    for fold in (True, False):
        q, s = _run(ops, x, torch.zeros(768), _signs(768, 9), 256, fold)
        assert int(q.abs().max()) == 0 and bool((s == 1).all())
        gamma = torch.tensor([-1.0, 0.0, 2.0]).repeat(256)
        _assert_oracle(ops, x, gamma, _signs(768, 9), 256, fold)


def test_rejections(ops):
    x = torch.zeros((3, 768), device=DEV)
    gamma = torch.ones(768, device=DEV)
    signs = torch.ones(768, dtype=torch.int8, device=DEV)
    with pytest.raises(TypeError, match="shift"):
        ops.rms_quantize(x, gamma, signs, shift=torch.zeros(768, device=DEV))
    with pytest.raises(NotImplementedError, match="register-resident"):
        ops.rms_quantize(torch.zeros((2, 65536), device=DEV), torch.ones(65536, device=DEV),
                         torch.ones(65536, dtype=torch.int8, device=DEV))
