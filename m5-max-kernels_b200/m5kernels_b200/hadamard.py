"""FP32 signed block Hadamard rotation X D H on B200 (twin of m5kernels.hadamard).

Mirrors src/m5kernels/hadamard.py:33-77: one shared int8 sign vector of +-1
applied before a normalized, block-diagonal Sylvester H; powers of two from
32 through 1024; K divisible by the block size; no padding.  The butterflies
run in FP32 (strides 1..B/2 in increasing order) and the result is scaled by
fp32(1/sqrt(B)) once at the end.
"""

from __future__ import annotations

from numbers import Integral

import torch

from . import _lib
from ._lib import check, ptr

SUPPORTED_BLOCK_SIZES = (32, 64, 128, 256, 512, 1024)
FLOAT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def validate_block(block_size, k):
    if (isinstance(block_size, bool) or not isinstance(block_size, Integral) or block_size <= 0
            or block_size & (block_size - 1)):
        raise ValueError("block_size must be a positive integer power of two")
    if int(block_size) not in SUPPORTED_BLOCK_SIZES:
        raise NotImplementedError("supported block sizes are powers of two from 32 through 1024")
    if k % int(block_size):
        raise NotImplementedError("K must be divisible by block_size; padding is not implicit")
    return int(block_size)


def validate_signs(signs, k):
    if signs is None:
        return None
    if tuple(signs.shape) != (k,) or signs.dtype != torch.int8:
        raise ValueError("signs must be an int8 vector of length K containing only +/-1")
    return signs.contiguous()


def rotate(x: torch.Tensor, block_size: int, signs: torch.Tensor, implementation: str = "cuda"):
    """Return FP32 X D H for nonempty X[rows, K] (bf16 / fp16 / fp32)."""
    if implementation not in ("cuda", "cuda-b200"):
        raise ValueError(f"unknown Hadamard implementation: {implementation}")
    if x.dim() != 2 or 0 in x.shape:
        raise ValueError("input must have nonempty shape [rows, K]")
    if x.dtype not in FLOAT_DTYPES:
        raise ValueError("input dtype must be float16, bfloat16 or float32")
    rows, k = x.shape
    block = validate_block(block_size, k)
    if signs is None:
        raise ValueError("signs must be an int8 vector of length K containing only +/-1")
    signs = validate_signs(signs, k)
    dev = _lib.require_cuda(x, signs)
    x = x.contiguous()
    y = torch.empty((rows, k), dtype=torch.float32, device=dev)
    check(_lib.lib().m5b_rotate(ptr(x), _lib.DTYPE_CODE[x.dtype], rows, k, block, ptr(signs),
                                ptr(y), _lib.stream_handle(dev)))
    return y


def hadamard_quantize(x: torch.Tensor, block_size: int, signs, mode: str = "int8"):
    """quantize(rotate(x), mode) in one pass (bit-identical to the two calls).

    The online activation preparation of src/m5kernels/hadamard_gemm.py:65-66.
    """
    if mode not in ("int8", "fp8"):
        raise NotImplementedError("rotation + quantization emits int8 or fp8 (E4M3)")
    if x.dim() != 2 or 0 in x.shape:
        raise ValueError("input must have nonempty shape [rows, K]")
    if x.dtype not in FLOAT_DTYPES:
        raise ValueError("input dtype must be float16, bfloat16 or float32")
    rows, k = x.shape
    block = validate_block(block_size, k)
    signs = validate_signs(signs, k)
    dev = _lib.require_cuda(x, signs)
    x = x.contiguous()
    q = torch.empty((rows, k), dtype=torch.int8 if mode == "int8" else torch.uint8, device=dev)
    s = torch.empty((rows,), dtype=torch.float32, device=dev)
    check(_lib.lib().m5b_hadamard_quantize(ptr(x), _lib.DTYPE_CODE[x.dtype], rows, k, block,
                                           ptr(signs), _lib.MODE[mode], ptr(q), ptr(s),
                                           _lib.stream_handle(dev)))
    return q, s
