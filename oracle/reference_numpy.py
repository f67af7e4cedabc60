"""Float64 NumPy restatement of the reference project's CPU references.

TEST INFRASTRUCTURE ONLY: tests/, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` leg of bench.py use this module as the checker.  The product
path (m5kernels_b200) never imports it.

Each function restates one reference function of 9Tempest/m5-max-kernels,
cited by file:line, with the same semantics (ideal float64 arithmetic with the
explicit rounding boundaries the reference defines).  They are pinned against
vectors produced by the reference itself (tests/golden/, see make_golden.py).
"""

from __future__ import annotations

import numpy as np

# --------------------------------------------------------------------- E4M3


def fp8_decode(codes) -> np.ndarray:
    """OCP E4M3 ("fn") bits -> float32; 0x7F / 0xFF are NaN.

    Restates src/m5kernels/numerics.py:6-14.
    """
    c = np.asarray(codes, dtype=np.uint8).astype(np.int64)
    negative = (c & 0x80) != 0
    exponent = (c >> 3) & 0xF
    mantissa = c & 0x7
    normal = (8 + mantissa) * np.exp2(exponent - 10.0)  # (1 + m/8) * 2^(e-7)
    subnormal = mantissa * 2.0**-9
    magnitude = np.where(exponent == 0, subnormal, normal)
    value = np.where(negative, -magnitude, magnitude)
    value = np.where((exponent == 15) & (mantissa == 7), np.nan, value)
    return value.astype(np.float32)


_E4M3_POSITIVE = fp8_decode(np.arange(127, dtype=np.uint8)).astype(np.float64)


def fp8_encode(x) -> np.ndarray:
    """Nearest finite E4M3 code, ties to the even code, saturating at 448.

    Restates src/m5kernels/numerics.py:17-26 (search over the positive
    codebook 0..126; the sign bit comes from signbit, so -0.0 -> 0x80).
    """
    x = np.asarray(x, dtype=np.float32)
    mag = np.minimum(np.abs(x).astype(np.float64), 448.0)
    upper = np.minimum(np.searchsorted(_E4M3_POSITIVE, mag), 126)
    lower = np.maximum(upper - 1, 0)
    below = mag - _E4M3_POSITIVE[lower]
    above = _E4M3_POSITIVE[upper] - mag
    take_lower = (below < above) | ((below == above) & (lower % 2 == 0))
    code = np.where(take_lower, lower, upper).astype(np.uint8)
    return code | np.where(np.signbit(x), np.uint8(0x80), np.uint8(0))


# --------------------------------------------------------------- quantizers


def quantize_reference(x, mode: str):
    """Per-row symmetric quantization in float32 arithmetic.

    Restates src/m5kernels/numerics.py:29-46: scale = peak/127 (int8) or
    peak/448 (fp8), zero rows scale 1, codes clip(rint(x/scale), +-127) or
    fp8_encode(x/scale); mxint8 uses 32-element power-of-two blocks.
    """
    x = np.asarray(x, dtype=np.float32)
    if not np.isfinite(x).all():
        raise ValueError("quantization input must be finite")
    if mode == "mxint8":
        if x.shape[-1] % 32:
            raise ValueError("K must be divisible by 32")
        blocks = x.reshape(*x.shape[:-1], -1, 32)
        peak = np.abs(blocks).max(axis=-1, keepdims=True)
        tiny = np.finfo(np.float32).tiny
        exponent = np.clip(np.floor(np.log2(np.maximum(peak, tiny))) - 6, -127, 127)
        exponent = np.where(peak == 0, 0, exponent)
        codes = np.clip(np.rint(blocks / np.exp2(exponent)), -127, 127).astype(np.int8)
        return codes.reshape(x.shape), (exponent[..., 0] + 127).astype(np.uint8)
    qmax = np.float32(448.0 if mode == "fp8" else 127.0)
    peak = np.abs(x).max(axis=-1, keepdims=True)
    scale = np.where(peak == 0, np.float32(1.0), peak / qmax).astype(np.float32)
    z = x / scale
    if mode == "fp8":
        codes = fp8_encode(z)
    else:
        codes = np.clip(np.rint(z), -127, 127).astype(np.int8)
    return codes, scale[..., 0]


def dequantize(q, s, mode: str) -> np.ndarray:
    """Restates src/m5kernels/numerics.py:49-54."""
    if mode == "mxint8":
        q = np.asarray(q)
        blocks = q.reshape(*q.shape[:-1], -1, 32).astype(np.float32)
        factor = np.exp2(np.asarray(s).astype(np.int32) - 127)[..., None]
        return (blocks * factor).reshape(q.shape)
    decoded = fp8_decode(q) if mode == "fp8" else np.asarray(q).astype(np.float32)
    return decoded * np.asarray(s)[..., None]


def metrics(actual, reference) -> dict:
    """Relative L2 / max abs / RMSE / cosine.  Restates numerics.py:57-75."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(reference, dtype=np.float64)
    if a.shape != r.shape:
        raise ValueError("reference shape mismatch")
    if not (np.isfinite(a).all() and np.isfinite(r).all()):
        return {"finite": False, "relative_l2": None, "max_abs": None, "rmse": None, "cosine": None}
    d = a - r
    rn, an = np.linalg.norm(r), np.linalg.norm(a)
    cosine = float(np.dot(a.ravel(), r.ravel()) / max(rn * an, 1e-30)) if rn else float(an == 0)
    return {
        "finite": True,
        "relative_l2": float(np.linalg.norm(d) / max(rn, 1e-30)),
        "max_abs": float(np.abs(d).max()) if d.size else 0.0,
        "rmse": float(np.sqrt(np.mean(d * d))) if d.size else 0.0,
        "cosine": cosine,
    }


def sample_indices(length: int, count: int = 32) -> np.ndarray:
    """Evenly spaced unique indices.  Restates numerics.py:78-79."""
    return np.unique(np.linspace(0, length - 1, min(length, count), dtype=int))


# ----------------------------------------------------------------- Hadamard


def hadamard_signs(k: int, seed) -> np.ndarray:
    """Shared +-1 int8 signs from PCG64(seed).  Restates hadamard_reference.py:19-23."""
    if isinstance(k, bool) or not isinstance(k, (int, np.integer)) or k <= 0:
        raise ValueError("K must be a positive integer")
    draws = np.random.Generator(np.random.PCG64(seed)).integers(0, 2, size=int(k), dtype=np.int8)
    return (2 * draws - 1).astype(np.int8)


def block_hadamard_reference(x, block_size: int, signs=None) -> np.ndarray:
    """X D H in float64: signs, 1/sqrt(B) scaling, then natural-order butterflies.

    Restates src/m5kernels/hadamard_reference.py:26-68 (scaling before the
    butterflies; blocks are contiguous along K; no padding).
    """
    if isinstance(block_size, bool) or not isinstance(block_size, (int, np.integer)) or block_size <= 0:
        raise ValueError("block_size must be a positive integer")
    if block_size & (block_size - 1):
        raise ValueError("block_size must be a power of two")
    x = np.asarray(x)
    if x.ndim != 2 or 0 in x.shape:
        raise ValueError("input must have nonempty shape [rows, K]")
    if x.shape[1] % block_size:
        raise ValueError("K must be divisible by block_size")
    y = np.array(x, dtype=np.float64, order="C", copy=True)
    if not np.isfinite(y).all():
        raise ValueError("input must be finite")
    if signs is not None:
        signs = np.asarray(signs)
        if signs.shape != (x.shape[1],) or not np.isin(signs, (-1, 1)).all():
            raise ValueError("signs must contain only -1 and +1 with length K")
        y *= signs
    y /= np.sqrt(float(block_size))
    view = y.reshape(-1, block_size)
    half = 1
    while half < block_size:
        pairs = view.reshape(-1, 2 * half)
        lo = pairs[:, :half].copy()
        hi = pairs[:, half:].copy()
        pairs[:, :half] = lo + hi
        pairs[:, half:] = lo - hi
        half *= 2
    return y


# -------------------------------------------------------------- norm / AdaLN


def norm_modulate_reference(x, gamma, scale, shift, *, norm="rms", eps=1e-5) -> np.ndarray:
    """norm(X) * gamma * (1 + scale) + shift in float64.

    Restates src/m5kernels/norm_hadamard_reference.py:24-64: RMS uses the row
    mean square; LayerNorm centers (after subtracting the first column, which
    keeps constant rows exact) and uses the population variance; epsilon is
    inside the square root.
    """
    if norm not in ("rms", "layer"):
        raise ValueError("norm must be 'rms' or 'layer'")
    if isinstance(eps, bool) or not np.isreal(eps) or not np.isfinite(eps) or eps <= 0:
        raise ValueError("eps must be a positive finite real scalar")
    x = np.asarray(x, dtype=np.float64)
    gamma, scale, shift = (np.asarray(v, dtype=np.float64) for v in (gamma, scale, shift))
    centered = x
    if norm == "layer":
        centered = x - x[:, :1]
        centered = centered - centered.mean(axis=1, keepdims=True)
    moment = (centered * centered).mean(axis=1, keepdims=True)
    return centered / np.sqrt(moment + float(eps)) * gamma * (1.0 + scale) + shift


def norm_hadamard_quantize_reference(x, gamma, scale, shift, block_size, signs=None, *, norm="rms", eps=1e-5):
    """Ideal modulation -> rotation -> per-row INT8 (float64 scales).

    Restates src/m5kernels/norm_hadamard_reference.py:67-94.
    """
    modulated = norm_modulate_reference(x, gamma, scale, shift, norm=norm, eps=eps)
    rotated = block_hadamard_reference(modulated, block_size, signs)
    peak = np.abs(rotated).max(axis=1)
    scales = np.where(peak == 0, 1.0, peak / 127.0)
    codes = np.clip(np.rint(rotated / scales[:, None]), -127, 127).astype(np.int8)
    return {
        "modulated": modulated,
        "rotated": rotated,
        "quantized": codes,
        "scales": scales,
        "dequantized": codes.astype(np.float64) * scales[:, None],
    }


def gated_residual_reference(residual, branch, gate, *, row_map=None) -> np.ndarray:
    """residual + gate[row_map] * branch in float64.

    Restates src/m5kernels/gated_residual_reference.py:21-60.
    """
    r = np.asarray(residual, dtype=np.float64)
    b = np.asarray(branch, dtype=np.float64)
    g = np.asarray(gate, dtype=np.float64)
    if g.ndim == 2:
        if row_map is None:
            raise ValueError("gate table requires row_map")
        g = g[np.asarray(row_map)]
    elif row_map is not None:
        raise ValueError("row_map is only supported with a gate table")
    return r + g * b


# ------------------------------------------------------------------ Q/K RoPE


def bf16_round_reference(value) -> np.ndarray:
    """float64 -> float32 -> bf16 (nearest even), returned as float64.

    Restates src/m5kernels/qk_rope_reference.py:24-42.
    """
    f32 = np.array(value, dtype=np.float32, order="C", copy=True)
    bits = f32.view(np.uint32)
    bits = (bits + np.uint32(0x7FFF) + ((bits >> 16) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return bits.view(np.float32).astype(np.float64)


def qk_rope_reference(projected, gamma, cos, sin, *, epsilon=1e-5, projection_bf16=True,
                      norm_bf16=False, output_bf16=True) -> dict:
    """Per-(row, head) RMSNorm over all D channels, gamma, split-half RoPE.

    Restates src/m5kernels/qk_rope_reference.py:45-134: projected is
    [M, H, D]; pairs (j, j + R) for j < R rotate by (cos, sin)[row, j];
    channels >= 2R are normalized but not rotated; the output is head-major
    [H, M, D].
    """
    p = np.asarray(projected, dtype=np.float64)
    p = bf16_round_reference(p) if projection_bf16 else p.copy()
    gamma = np.asarray(gamma, dtype=np.float64)
    cos = np.asarray(cos, dtype=np.float64)
    sin = np.asarray(sin, dtype=np.float64)
    inverse = 1.0 / np.sqrt((p * p).mean(axis=-1) + float(epsilon))
    normalized = p * inverse[..., None] * gamma
    if norm_bf16:
        normalized = bf16_round_reference(normalized)
    half = cos.shape[1]
    rotated = normalized.copy()
    lo = normalized[..., :half]
    hi = normalized[..., half:2 * half]
    c = cos[:, None, :]
    s = sin[:, None, :]
    rotated[..., :half] = lo * c - hi * s
    rotated[..., half:2 * half] = hi * c + lo * s
    out = bf16_round_reference(rotated) if output_bf16 else rotated
    return {
        "projected": p,
        "inverse_rms": inverse,
        "normalized": normalized,
        "rotated": rotated,
        "output": np.ascontiguousarray(out.transpose(1, 0, 2)),
    }


# ------------------------------------------------------- RMS scale folding


def rms_quantize_reference(x, gamma, signs=None, block_size=1, eps=1e-5) -> dict:
    """RMS(X) * gamma, signed block Hadamard, per-row INT8 with folded scales.

    Restates src/m5kernels/rms_quant_reference.py:24-89 in float64:
    r = 1 / sqrt(mean(X^2) + eps) from the ORIGINAL rows; U = (X * gamma) D H;
    codes rint(U / (peak(U) / 127)) clipped to +-127 (nearest even), scales
    peak(U) / 127 * r; a row with peak(U) == 0 gets codes 0 and scale 1.  The
    positive factor r changes the scales only, never the codes.
    """
    if isinstance(eps, bool) or not np.isscalar(eps) or np.iscomplexobj(eps):
        raise ValueError("eps must be a positive finite real scalar")
    if not np.isfinite(eps) or eps <= 0:
        raise ValueError("eps must be a positive finite real scalar")
    xv, gv = np.asarray(x), np.asarray(gamma)
    for name, value in (("input", xv), ("gamma", gv)):
        if np.iscomplexobj(value):
            raise ValueError(f"{name} must be real")
    xv = np.asarray(xv, dtype=np.float64)
    gv = np.asarray(gv, dtype=np.float64)
    if not np.isfinite(xv).all():
        raise ValueError("input must be finite")
    if not np.isfinite(gv).all():
        raise ValueError("gamma must be finite")
    if xv.ndim != 2 or 0 in xv.shape:
        raise ValueError("input must have nonempty shape [M,K]")
    if gv.shape != (xv.shape[1],):
        raise ValueError("gamma must have shape [K]")
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        moment = np.mean(xv * xv, axis=1)
        inverse_rms = 1.0 / np.sqrt(moment + float(eps))
        weighted = xv * gv
    if (not np.isfinite(moment).all() or not np.isfinite(inverse_rms).all()
            or not np.all(inverse_rms > 0) or not np.isfinite(weighted).all()):
        raise ValueError("RMS or gamma multiplication exceeds finite float64 range")
    unscaled = block_hadamard_reference(weighted, block_size, signs)
    peak = np.max(np.abs(unscaled), axis=1)
    nonzero = peak != 0
    unscaled_scales = np.where(nonzero, peak / 127.0, 1.0)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        normalized_rotated = unscaled * inverse_rms[:, None]
        scales = np.where(nonzero, unscaled_scales * inverse_rms, 1.0)
    codes = np.clip(np.rint(unscaled / unscaled_scales[:, None]), -127, 127).astype(np.int8)
    return {
        "normalized_rotated": normalized_rotated,
        "quantized": codes,
        "scales": scales,
        "dequantized": codes.astype(np.float64) * scales[:, None],
        "unscaled_rotated": unscaled,
        "inverse_rms": inverse_rms,
        "unscaled_scales": unscaled_scales,
    }
