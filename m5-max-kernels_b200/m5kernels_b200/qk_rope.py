"""Head-aligned Q/K projection + per-head RMSNorm + split-half RoPE on B200.

Twin of m5kernels.qk_rope.projection_qk_rope (src/m5kernels/qk_rope.py:120-182).
One tcgen05 GEMM tile of 128 x 128 is exactly one head of 128 rows; its
epilogue rounds the projection to BF16, computes the row's RMS over the
head's 128 channels, applies gamma and rotates the pairs (j, j + R) for j < R,
and writes the head-major [H, M, 128] BF16 output.  Boundaries: BF16
projection, FP32 RMS/gamma/RoPE, BF16 output (no BF16 norm intermediate).

`projection_qkv_rope` runs the grouped Q/K/V weight layout [head, stream, 128]
of the reference's H3 integration in one GEMM with three head-major outputs.

`qk_norm_rope` is the staged comparator (src/m5kernels/qk_rope.py:185-203):
the same post-processing applied to a stored BF16 projection, bit-identical to
the fused epilogue, so gemm(..., bf16) -> qk_norm_rope == projection_qk_rope.
"""

from __future__ import annotations

import math
import struct
from numbers import Integral, Real

import torch

from . import _lib
from ._lib import check, ptr

HEAD_DIM = 128


def _epsilon(epsilon):
    if (isinstance(epsilon, bool) or not isinstance(epsilon, Real) or not math.isfinite(epsilon)
            or epsilon <= 0):
        raise ValueError("epsilon must be a positive finite real scalar")
    try:
        value = struct.unpack("=f", struct.pack("=f", float(epsilon)))[0]
    except OverflowError:
        raise ValueError("epsilon must remain finite and positive in float32") from None
    if not math.isfinite(value) or value <= 0:
        raise ValueError("epsilon must remain finite and positive in float32")
    return value


def _validate_norm(m, n, gamma, cos, sin, epsilon):
    if m <= 0 or n <= 0 or n % HEAD_DIM:
        raise ValueError("projection must have nonempty [M,N] shape with whole 128-wide heads")
    if tuple(gamma.shape) != (HEAD_DIM,) or gamma.dtype != torch.bfloat16:
        raise ValueError("gamma must be a shared bfloat16 vector of length 128")
    if cos.dim() != 2 or cos.shape[0] != m or not 1 <= cos.shape[1] <= HEAD_DIM // 2:
        raise ValueError("cos must have shape [M,rope_half] with rope_half in [1,64]")
    if tuple(sin.shape) != tuple(cos.shape) or cos.dtype != torch.bfloat16 or sin.dtype != torch.bfloat16:
        raise ValueError("cos and sin must have matching bfloat16 [M,rope_half] shapes")
    return cos.shape[1], _epsilon(epsilon)


def projection_qk_rope(a, b, gamma, cos, sin, mode="int8", tile=(32, 128, 4, 1), *,
                       a_scales=None, b_scales=None, epsilon=1e-5):
    """Return BF16 [heads, M, 128] Q or K after projection, RMSNorm and RoPE."""
    if mode not in ("int8", "bf16"):
        raise NotImplementedError("Q/K projection fusion supports INT8 or BF16 only")
    if a.dim() != 2 or b.dim() != 2 or 0 in a.shape or 0 in b.shape:
        raise ValueError("A and B must be nonempty matrices")
    m, k = a.shape
    n, kb = b.shape
    if k != kb:
        raise ValueError("K mismatch")
    expected = torch.int8 if mode == "int8" else torch.bfloat16
    if a.dtype != expected or b.dtype != expected:
        raise ValueError(f"A and B must both have {mode} dtype")
    if mode == "int8":
        if k > 131071:
            raise NotImplementedError("INT32 worst-case overflow bound exceeded for signed INT8")
        if (a_scales is None or b_scales is None or tuple(a_scales.shape) != (m,)
                or tuple(b_scales.shape) != (n,) or a_scales.dtype != torch.float32
                or b_scales.dtype != torch.float32):
            raise ValueError("INT8 requires float32 a_scales[M] and b_scales[N]")
    elif a_scales is not None or b_scales is not None:
        raise ValueError("BF16 projection does not accept quantization scales")
    rope_half, eps = _validate_norm(m, n, gamma, cos, sin, epsilon)
    if not isinstance(tile, (tuple, list)) or len(tile) != 4:
        raise ValueError("tile must contain TM, TN, SIMD groups and M swizzle")
    dev = _lib.require_cuda(a, b, gamma, cos, sin, a_scales, b_scales)
    elem = 1 if mode == "int8" else 2
    pad = (-k) % (16 // elem)
    a, b = a.contiguous(), b.contiguous()
    if pad:
        a = torch.nn.functional.pad(a, (0, pad))
        b = torch.nn.functional.pad(b, (0, pad))
    gamma, cos, sin = gamma.contiguous(), cos.contiguous(), sin.contiguous()
    a_scales = a_scales.contiguous() if a_scales is not None else None
    b_scales = b_scales.contiguous() if b_scales is not None else None
    out = torch.empty((n // HEAD_DIM, m, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    lib = _lib.lib()
    from .linear import gemm_workspace  # split-K workspace for the shapes that split

    ws = gemm_workspace(dev, int(lib.m5b_gemm_workspace_bytes(m, n, a.shape[1], _lib.MODE[mode])))
    check(lib.m5b_projection_qk_rope_ex(
        ptr(a), ptr(b), m, n, a.shape[1], _lib.MODE[mode], ptr(a_scales), ptr(b_scales),
        ptr(gamma), ptr(cos), ptr(sin), rope_half, eps, ptr(out), ptr(ws),
        0 if ws is None else ws.numel(), _lib.stream_handle(dev)))
    return out


def projection_qkv_rope(a, b, gamma_q, gamma_k, cos, sin, mode="int8", *, a_scales=None,
                        b_scales=None, epsilon=1e-5):
    """Grouped Q/K/V projection: return BF16 (q, k, v), each [heads, M, 128].

    b holds the native grouped weight order [heads, 3, 128, K] (flattened to
    [heads*384, K]): per head the Q, K and V channel blocks.  Q and K get
    per-head RMSNorm with their own gamma and split-half RoPE; V is the BF16
    projection in head-major layout.  Counterpart of the grouped QKV path of
    the reference's H3 integration (integrations/h3/qkv-candidate.md:30-43,
    qkv_reference.h:15-36).
    """
    if mode not in ("int8", "bf16"):
        raise NotImplementedError("grouped Q/K/V projection supports INT8 or BF16 only")
    if a.dim() != 2 or b.dim() != 2 or 0 in a.shape or 0 in b.shape:
        raise ValueError("A and B must be nonempty matrices")
    m, k = a.shape
    n, kb = b.shape
    if k != kb:
        raise ValueError("K mismatch")
    if n % (3 * HEAD_DIM):
        raise ValueError("grouped weights must have [heads, 3, 128, K] rows")
    heads = n // (3 * HEAD_DIM)
    expected = torch.int8 if mode == "int8" else torch.bfloat16
    if a.dtype != expected or b.dtype != expected:
        raise ValueError(f"A and B must both have {mode} dtype")
    if mode == "int8":
        if k > 131071:
            raise NotImplementedError("INT32 worst-case overflow bound exceeded for signed INT8")
        if (a_scales is None or b_scales is None or tuple(a_scales.shape) != (m,)
                or tuple(b_scales.shape) != (n,) or a_scales.dtype != torch.float32
                or b_scales.dtype != torch.float32):
            raise ValueError("INT8 requires float32 a_scales[M] and b_scales[N]")
    elif a_scales is not None or b_scales is not None:
        raise ValueError("BF16 projection does not accept quantization scales")
    rope_half, eps = _validate_norm(m, HEAD_DIM, gamma_q, cos, sin, epsilon)
    if tuple(gamma_k.shape) != (HEAD_DIM,) or gamma_k.dtype != torch.bfloat16:
        raise ValueError("gamma must be a shared bfloat16 vector of length 128")
    dev = _lib.require_cuda(a, b, gamma_q, gamma_k, cos, sin, a_scales, b_scales)
    elem = 1 if mode == "int8" else 2
    pad = (-k) % (16 // elem)
    a, b = a.contiguous(), b.contiguous()
    if pad:
        a = torch.nn.functional.pad(a, (0, pad))
        b = torch.nn.functional.pad(b, (0, pad))
    gamma_q, gamma_k = gamma_q.contiguous(), gamma_k.contiguous()
    cos, sin = cos.contiguous(), sin.contiguous()
    a_scales = a_scales.contiguous() if a_scales is not None else None
    b_scales = b_scales.contiguous() if b_scales is not None else None
    outs = [torch.empty((heads, m, HEAD_DIM), dtype=torch.bfloat16, device=dev) for _ in range(3)]
    check(_lib.lib().m5b_projection_qkv_rope(
        ptr(a), ptr(b), m, heads, a.shape[1], _lib.MODE[mode], ptr(a_scales), ptr(b_scales),
        ptr(gamma_q), ptr(gamma_k), ptr(cos), ptr(sin), rope_half, eps, ptr(outs[0]),
        ptr(outs[1]), ptr(outs[2]), _lib.stream_handle(dev)))
    return tuple(outs)


def grouped_qkv_weights(wq, wk, wv):
    """Interleave separate [H*128, K] Q, K, V weights into the grouped [H*3*128, K] order."""
    if not (wq.shape == wk.shape == wv.shape) or wq.dim() != 2 or wq.shape[0] % HEAD_DIM:
        raise ValueError("Q, K and V weights must share one [H*128, K] shape")
    h, k = wq.shape[0] // HEAD_DIM, wq.shape[1]
    return torch.stack([w.reshape(h, HEAD_DIM, k) for w in (wq, wk, wv)], dim=1).reshape(-1, k)


def qk_norm_rope(projected, gamma, cos, sin, *, epsilon=1e-5, threads=128):
    """Standalone post-process from BF16 [M, N] to BF16 [heads, M, 128]."""
    if not isinstance(projected, torch.Tensor) or projected.dim() != 2 or projected.dtype != torch.bfloat16:
        raise ValueError("projected must be a bfloat16 [M,N] matrix")
    m, n = projected.shape
    rope_half, eps = _validate_norm(m, n, gamma, cos, sin, epsilon)
    if isinstance(threads, bool) or not isinstance(threads, Integral):
        raise ValueError("threads must be an integer")
    if threads not in (128, 256):
        raise NotImplementedError("standalone Q/K normalization supports 128 or 256 threads")
    dev = _lib.require_cuda(projected, gamma, cos, sin)
    projected = projected.contiguous()
    if projected.data_ptr() % 16:
        projected = projected.clone()
    gamma, cos, sin = gamma.contiguous(), cos.contiguous(), sin.contiguous()
    out = torch.empty((n // HEAD_DIM, m, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    check(_lib.lib().m5b_qk_norm_rope(
        ptr(projected), m, n, ptr(gamma), ptr(cos), ptr(sin), rope_half, eps, ptr(out),
        _lib.stream_handle(dev)))
    return out


def rope_tables(m: int, rope_half: int = 64, theta: float = 10000.0, *, positions=None,
                device=None):
    """BF16 cos/sin tables [M, R] for split-half RoPE.

    angle[p, j] = p * theta ** (-j / R) for j < R (positions 0..M-1 unless
    given), evaluated in float64 and rounded to BF16 once.  This is the table
    definition the B200 workloads use (the reference takes cos/sin as inputs).
    """
    pos = torch.arange(m, dtype=torch.float64) if positions is None else positions.double().cpu()
    inv_freq = theta ** (-torch.arange(rope_half, dtype=torch.float64) / rope_half)
    ang = pos[:, None] * inv_freq[None, :]
    cos = torch.cos(ang).to(torch.float32).to(torch.bfloat16)
    sin = torch.sin(ang).to(torch.float32).to(torch.bfloat16)
    if device is not None:
        cos, sin = cos.to(device), sin.to(device)
    return cos, sin
