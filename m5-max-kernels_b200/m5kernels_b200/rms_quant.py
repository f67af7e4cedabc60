"""RMS dynamic INT8 preparation with the inverse RMS folded into row scales, on B200.

Twin of m5kernels.rms_quant (src/m5kernels/rms_quant.py:41-117): RMS
statistics come from the original rows, gamma is a shared FP32 [K] vector
(possibly a pre-combined gamma * (1 + AdaLN scale)), there is no additive
shift and no rounding to the input dtype after normalization.

    fold_scale=True : u = (x * gamma) D H; codes rint(127 * u / peak(u));
                      scale = peak(u) * r / 127 with r = 1 / sqrt(mean(x^2) + eps)
    fold_scale=False: u = ((x * r) * gamma) D H; scale = peak(u) / 127

A row whose u is all zero gets codes 0 and scale 1.  `threads` and `tag` are
Metal launch knobs, accepted and validated for signature compatibility; the
CUDA kernel keeps each row register-resident and chooses its own CTA size.
"""

from __future__ import annotations

import math
import re
import struct
from numbers import Integral, Real

import torch

from . import _lib
from ._lib import check, ptr

BLOCK_SIZES = (1, 32, 64, 128, 256, 512, 1024)
FLOAT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _validate(x, gamma, signs, block_size, threads, fold_scale, epsilon, tag):
    if x.dim() != 2 or 0 in x.shape:
        raise ValueError("input must have nonempty shape [M,K]")
    if x.dtype not in FLOAT_DTYPES:
        raise ValueError("input dtype must be float16, bfloat16 or float32")
    k = x.shape[1]
    if tuple(gamma.shape) != (k,) or gamma.dtype != torch.float32:
        raise ValueError("gamma must be a float32 vector of length K")
    if tuple(signs.shape) != (k,) or signs.dtype != torch.int8:
        raise ValueError("signs must be an int8 vector of length K containing only +/-1")
    if (isinstance(block_size, bool) or not isinstance(block_size, Integral) or block_size <= 0
            or block_size & (block_size - 1)):
        raise ValueError("block_size must be a positive integer power of two")
    if int(block_size) not in BLOCK_SIZES:
        raise NotImplementedError("supported blocks are 1 and powers of two from 32 through 1024")
    if k % int(block_size):
        raise NotImplementedError("K must be divisible by block_size; padding is not implicit")
    if isinstance(threads, bool) or not isinstance(threads, Integral):
        raise ValueError("threads must be an integer")
    if threads not in (128, 256, 512):
        raise NotImplementedError("supported threadgroup sizes are 128, 256 and 512")
    if not isinstance(fold_scale, bool):
        raise ValueError("fold_scale must be a boolean")
    if (isinstance(epsilon, bool) or not isinstance(epsilon, Real) or not math.isfinite(epsilon)
            or epsilon <= 0):
        raise ValueError("epsilon must be a positive finite real scalar")
    try:
        eps32 = struct.unpack("=f", struct.pack("=f", float(epsilon)))[0]
    except OverflowError:
        raise ValueError("epsilon must remain finite and positive in float32") from None
    if not math.isfinite(eps32) or eps32 <= 0:
        raise ValueError("epsilon must remain finite and positive in float32")
    if not isinstance(tag, str) or re.fullmatch(r"[A-Za-z_][A-Za-z_0-9]*", tag) is None:
        raise ValueError("tag must be a valid nonempty identifier")
    return int(block_size), eps32


def rms_quantize(x, gamma, signs, block_size=1, *, threads=256, fold_scale=True, epsilon=1e-5,
                 tag="default"):
    """Return per-row INT8 codes [M,K] and FP32 scales [M] of RMS(x) * gamma * D H."""
    block, eps32 = _validate(x, gamma, signs, block_size, threads, fold_scale, epsilon, tag)
    dev = _lib.require_cuda(x, gamma, signs)
    x, gamma, signs = x.contiguous(), gamma.contiguous(), signs.contiguous()
    rows, k = x.shape
    q = torch.empty((rows, k), dtype=torch.int8, device=dev)
    s = torch.empty((rows,), dtype=torch.float32, device=dev)
    check(_lib.lib().m5b_rms_quantize(ptr(x), _lib.DTYPE_CODE[x.dtype], rows, k, ptr(gamma),
                                      ptr(signs), block, 1 if fold_scale else 0, eps32, ptr(q),
                                      ptr(s), _lib.stream_handle(dev)))
    return q, s
