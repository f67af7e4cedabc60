"""One-kernel normalization, modulation, block rotation and quantization on B200.

Also the staged comparators of the same module (src/m5kernels/norm_hadamard.py:
280-348): `gated_residual_add` (the R' update alone) and `unfused_norm` (norm +
modulation alone).  Each runs the fused kernels' FP32 operations in the same
order, so gated_residual_add -> fused_norm_hadamard_quantize equals the fused
gated kernel bit for bit, and unfused_norm -> hadamard_quantize equals
fused_norm_hadamard_quantize.

Twin of m5kernels.norm_hadamard (src/m5kernels/norm_hadamard.py:122-265):
the modulation contract is norm(X) * gamma * (1 + scale) + shift in FP32,
optionally rounded to X's dtype after the complete expression; signs are
applied after that rounding and before the normalized Hadamard butterflies;
codes are symmetric per-row INT8 (or E4M3, an extension) with scale
peak/127 (peak/448) and scale 1 for an all-zero row.

`threads`, `passes` and `tag` are accepted for signature compatibility: the
B200 kernel keeps each row register-resident (one read of HBM) and chooses
its own CTA size.
"""

from __future__ import annotations

import math
import re
from numbers import Integral, Real

import torch

from . import _lib
from ._lib import check, ptr
from .hadamard import validate_block, validate_signs

FLOAT_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _validate_common(x, gamma, scale, shift, norm, epsilon, round_output, threads, row_map):
    if x.dim() != 2 or 0 in x.shape:
        raise ValueError("input must have nonempty shape [rows, K]")
    if x.dtype not in FLOAT_DTYPES:
        raise ValueError("input dtype must be float16, bfloat16 or float32")
    k = x.shape[1]
    if tuple(gamma.shape) != (k,) or gamma.dtype not in FLOAT_DTYPES:
        raise ValueError("gamma must be a floating vector of length K")
    if row_map is None:
        if tuple(scale.shape) != (k,) or tuple(shift.shape) != tuple(scale.shape):
            raise ValueError("scale and shift must be vectors of length K without row_map")
    else:
        if (scale.dim() != 2 or 0 in scale.shape or scale.shape[1] != k
                or tuple(shift.shape) != tuple(scale.shape)):
            raise ValueError("mapped scale and shift must have matching nonempty shape [P,K]")
        if tuple(row_map.shape) != (x.shape[0],) or row_map.dtype != torch.int32:
            raise ValueError("row_map must be an int32 vector of length M")
    if scale.dtype not in FLOAT_DTYPES or shift.dtype not in FLOAT_DTYPES:
        raise ValueError("scale and shift must have floating dtype")
    if norm == "layernorm":
        norm = "layer"
    if norm not in ("rms", "layer"):
        raise ValueError("norm must be 'rms' or 'layer'")
    if isinstance(epsilon, bool) or not isinstance(epsilon, Real):
        raise ValueError("epsilon must be a positive finite real scalar")
    if not math.isfinite(epsilon) or epsilon <= 0:
        raise ValueError("epsilon must be a positive finite real scalar")
    if round_output not in ("input", "fp32"):
        raise ValueError("round_output must be 'input' or 'fp32'")
    if isinstance(threads, bool) or not isinstance(threads, Integral):
        raise ValueError("threads must be an integer")
    if threads not in (128, 256):
        raise NotImplementedError("supported threadgroup sizes are 128 and 256")
    return norm


def _validate_rotation(x, signs, block_size, passes, tag):
    block = validate_block(block_size, x.shape[1])
    signs = validate_signs(signs, x.shape[1])
    if signs is None:
        raise ValueError("signs must be an int8 vector of length K containing only +/-1")
    if passes not in ("one_read", "two_read"):
        raise ValueError("passes must be 'one_read' or 'two_read'")
    if not isinstance(tag, str) or re.fullmatch(r"[A-Za-z_][A-Za-z_0-9]*", tag) is None:
        raise ValueError("tag must be a valid nonempty identifier")
    return block, signs


def _out_mode(out):
    if out not in ("int8", "fp8"):
        raise NotImplementedError("the fused preparation emits int8 or fp8 (E4M3)")
    return out


def fused_norm_hadamard_quantize(x, gamma, scale, shift, signs, block_size=256, *, norm="rms",
                                 epsilon=1e-5, round_output="input", threads=256,
                                 passes="one_read", tag="default", row_map=None, out="int8"):
    """Return per-row (codes, fp32 scales) of quantize(modulate(norm(x)) D H)."""
    norm = _validate_common(x, gamma, scale, shift, norm, epsilon, round_output, threads, row_map)
    block, signs = _validate_rotation(x, signs, block_size, passes, tag)
    mode = _out_mode(out)
    dev = _lib.require_cuda(x, gamma, scale, shift, signs, row_map)
    x, gamma, scale, shift = (t.contiguous() for t in (x, gamma, scale, shift))
    row_map = row_map.contiguous() if row_map is not None else None
    rows, k = x.shape
    q = torch.empty((rows, k), dtype=torch.int8 if mode == "int8" else torch.uint8, device=dev)
    s = torch.empty((rows,), dtype=torch.float32, device=dev)
    code = _lib.DTYPE_CODE
    check(_lib.lib().m5b_fused_norm_hadamard_quantize(
        ptr(x), code[x.dtype], rows, k, ptr(gamma), code[gamma.dtype], ptr(scale),
        code[scale.dtype], ptr(shift), code[shift.dtype], ptr(row_map),
        scale.shape[0] if row_map is not None else 0, ptr(signs), block, _lib.NORM[norm],
        float(epsilon), 1 if round_output == "input" else 0, _lib.MODE[mode], ptr(q), ptr(s),
        _lib.stream_handle(dev)))
    return q, s


def _validate_gate(residual, branch, gate, gate_row_map):
    if residual.dim() != 2 or 0 in residual.shape:
        raise ValueError("residual must have nonempty shape [M,K]")
    if residual.dtype not in FLOAT_DTYPES:
        raise ValueError("residual must have floating dtype")
    if tuple(branch.shape) != tuple(residual.shape) or branch.dtype not in FLOAT_DTYPES:
        raise ValueError("branch must have the same shape as residual and floating dtype")
    if gate.dtype not in FLOAT_DTYPES:
        raise ValueError("gate must have floating dtype")
    if gate_row_map is None:
        if tuple(gate.shape) != (residual.shape[1],):
            raise ValueError("gate must be a vector of length K without gate_row_map")
    else:
        if gate.dim() != 2 or 0 in gate.shape or gate.shape[1] != residual.shape[1]:
            raise ValueError("mapped gate must have nonempty shape [P,K]")
        if tuple(gate_row_map.shape) != (residual.shape[0],) or gate_row_map.dtype != torch.int32:
            raise ValueError("gate_row_map must be an int32 vector of length M")


def fused_gated_residual_norm_hadamard_quantize(
        residual, branch, gate, gamma, scale, shift, signs, block_size=256, *, norm="rms",
        epsilon=1e-5, round_output="input", threads=256, passes="one_read", tag="default",
        gate_row_map=None, row_map=None, out="int8"):
    """Return (codes, scales, updated residual) in one kernel.

    R' = cast_R(float(R) + float(branch) * float(gate)) (one FP32 fused
    multiply-add, then round to the residual dtype) is written once and fed
    through the same normalization, modulation, rotation and quantization.
    Mirrors src/m5kernels/norm_hadamard.py:198-265.
    """
    _validate_gate(residual, branch, gate, gate_row_map)
    norm = _validate_common(residual, gamma, scale, shift, norm, epsilon, round_output, threads,
                            row_map)
    block, signs = _validate_rotation(residual, signs, block_size, passes, tag)
    mode = _out_mode(out)
    if branch.dtype != residual.dtype:
        raise NotImplementedError("branch and residual must share one dtype on cuda-b200")
    dev = _lib.require_cuda(residual, branch, gate, gamma, scale, shift, signs, row_map,
                            gate_row_map)
    residual, branch, gate, gamma, scale, shift = (
        t.contiguous() for t in (residual, branch, gate, gamma, scale, shift))
    row_map = row_map.contiguous() if row_map is not None else None
    gate_row_map = gate_row_map.contiguous() if gate_row_map is not None else None
    rows, k = residual.shape
    q = torch.empty((rows, k), dtype=torch.int8 if mode == "int8" else torch.uint8, device=dev)
    s = torch.empty((rows,), dtype=torch.float32, device=dev)
    r_out = torch.empty_like(residual)
    code = _lib.DTYPE_CODE
    check(_lib.lib().m5b_fused_gated_residual_norm_hadamard_quantize(
        ptr(residual), ptr(branch), code[residual.dtype], rows, k, ptr(gate), code[gate.dtype],
        ptr(gate_row_map), gate.shape[0] if gate_row_map is not None else 0, ptr(gamma),
        code[gamma.dtype], ptr(scale), code[scale.dtype], ptr(shift), code[shift.dtype],
        ptr(row_map), scale.shape[0] if row_map is not None else 0, ptr(signs), block,
        _lib.NORM[norm], float(epsilon), 1 if round_output == "input" else 0, _lib.MODE[mode],
        ptr(q), ptr(s), ptr(r_out), _lib.stream_handle(dev)))
    return q, s, r_out


def _validate_threads_tag(threads, tag):
    if isinstance(threads, bool) or not isinstance(threads, Integral):
        raise ValueError("threads must be an integer")
    if threads not in (128, 256):
        raise NotImplementedError("supported threadgroup sizes are 128 and 256")
    if not isinstance(tag, str) or re.fullmatch(r"[A-Za-z_][A-Za-z_0-9]*", tag) is None:
        raise ValueError("tag must be a valid nonempty identifier")


def gated_residual_add(residual, branch, gate, *, gate_row_map=None, threads=256, tag="default"):
    """Stage the gated residual update alone: cast_R(R + branch * gate[gate_row_map]).

    One FP32 fused multiply-add per element, then round to the residual dtype
    -- the R' that fused_gated_residual_norm_hadamard_quantize writes.  Twin of
    src/m5kernels/norm_hadamard.py:280-300.
    """
    _validate_gate(residual, branch, gate, gate_row_map)
    _validate_threads_tag(threads, tag)
    if branch.dtype != residual.dtype:
        raise NotImplementedError("branch and residual must share one dtype on cuda-b200")
    dev = _lib.require_cuda(residual, branch, gate, gate_row_map)
    residual, branch, gate = (t.contiguous() for t in (residual, branch, gate))
    gate_row_map = gate_row_map.contiguous() if gate_row_map is not None else None
    rows, k = residual.shape
    out = torch.empty_like(residual)
    code = _lib.DTYPE_CODE
    check(_lib.lib().m5b_gated_residual_add(
        ptr(residual), ptr(branch), code[residual.dtype], rows, k, ptr(gate), code[gate.dtype],
        ptr(gate_row_map), gate.shape[0] if gate_row_map is not None else 0, ptr(out),
        _lib.stream_handle(dev)))
    return out


def unfused_norm(x, gamma, scale, shift, *, norm="rms", epsilon=1e-5, round_output="input",
                 threads=256, row_map=None):
    """Return norm + modulation only, with the fused path's rounding contract.

    y = norm(x) * gamma * (1 + scale[row_map]) + shift[row_map] in FP32 with the
    statistics of fused_norm_hadamard_quantize; x's dtype when round_output is
    "input", else float32.  No rotation, no packing.  Twin of
    src/m5kernels/norm_hadamard.py:321-348.
    """
    norm = _validate_common(x, gamma, scale, shift, norm, epsilon, round_output, threads, row_map)
    dev = _lib.require_cuda(x, gamma, scale, shift, row_map)
    x, gamma, scale, shift = (t.contiguous() for t in (x, gamma, scale, shift))
    row_map = row_map.contiguous() if row_map is not None else None
    rows, k = x.shape
    dtype = x.dtype if round_output == "input" else torch.float32
    y = torch.empty((rows, k), dtype=dtype, device=dev)
    code = _lib.DTYPE_CODE
    check(_lib.lib().m5b_unfused_norm(
        ptr(x), code[x.dtype], rows, k, ptr(gamma), code[gamma.dtype], ptr(scale),
        code[scale.dtype], ptr(shift), code[shift.dtype], ptr(row_map),
        scale.shape[0] if row_map is not None else 0, _lib.NORM[norm], float(epsilon),
        1 if round_output == "input" else 0, ptr(y), _lib.stream_handle(dev)))
    return y
