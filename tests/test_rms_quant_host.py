"""Argument contract of the rms_quantize twin, checked on CPU (no kernel runs).

Mirrors the reference's rejections (tests/test_rms_quant_metal.py:160-181):
the same exception types and messages, raised before any device work; a
valid call with CPU tensors raises ExtensionMissing instead of falling back.
"""

import pytest
import torch

from m5kernels_b200 import rms_quantize
from m5kernels_b200._lib import ExtensionMissing


def _args(k=768):
    return torch.zeros((3, k)), torch.ones(k), torch.ones(k, dtype=torch.int8)


def test_no_shift_argument():
    x, gamma, signs = _args()
    with pytest.raises(TypeError, match="shift"):
        rms_quantize(x, gamma, signs, shift=torch.zeros(768))


@pytest.mark.parametrize("kwargs,error,match", [
    ({"block_size": 3}, ValueError, "power of two"),
    ({"block_size": 16}, NotImplementedError, "supported blocks"),
    ({"block_size": 512}, NotImplementedError, "divisible"),
    ({"threads": 32}, NotImplementedError, "threadgroup sizes"),
    ({"threads": 128.0}, ValueError, "integer"),
    ({"fold_scale": 1}, ValueError, "boolean"),
    ({"epsilon": 0}, ValueError, "positive finite"),
    ({"epsilon": True}, ValueError, "positive finite"),
    ({"epsilon": 1e-100}, ValueError, "finite and positive in float32"),
    ({"epsilon": 1e100}, ValueError, "finite and positive in float32"),
    ({"tag": "9bad"}, ValueError, "identifier"),
])
def test_explicit_rejections(kwargs, error, match):
    x, gamma, signs = _args()
    with pytest.raises(error, match=match):
        rms_quantize(x, gamma, signs, **kwargs)


def test_operand_contracts():
    x, gamma, signs = _args()
    with pytest.raises(ValueError, match="float32 vector"):
        rms_quantize(x, gamma.to(torch.bfloat16), signs)
    with pytest.raises(ValueError, match="int8 vector"):
        rms_quantize(x, gamma, torch.ones(768))
    with pytest.raises(ValueError, match="nonempty shape"):
        rms_quantize(torch.zeros((0, 768)), gamma, signs)
    with pytest.raises(ValueError, match="dtype"):
        rms_quantize(x.to(torch.int32), gamma, signs)


def test_cpu_tensors_do_not_fall_back():
    x, gamma, signs = _args()
    with pytest.raises(ExtensionMissing):
        rms_quantize(x, gamma, signs, 256)
