"""Float64 quality references used by the harness on sampled rows.

The reference harness checks each experiment against ideal float64
arithmetic with explicit rounding boundaries (src/m5kernels/engine.py:141-175,
norm_hadamard_gemm.py:86-133, qk_rope_experiment.py:266-296).  These helpers
are that check for the cuda-b200 backend: they only grade outputs on a few
sampled rows, they never produce an operator's result.
"""

from __future__ import annotations

import numpy as np
import torch


def _f64(t) -> np.ndarray:
    return t.detach().to("cpu", torch.float64).numpy()


def _bf16_round(x: np.ndarray) -> np.ndarray:
    """float64 -> float32 -> bf16 (nearest even) -> float64."""
    f32 = np.asarray(x, dtype=np.float32).copy()
    bits = f32.view(np.uint32)
    bits = (bits + np.uint32(0x7FFF) + ((bits >> 16) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return bits.view(np.float32).astype(np.float64)


def _fwht(x: np.ndarray, block: int) -> np.ndarray:
    y = np.array(x, dtype=np.float64, copy=True) / np.sqrt(block)
    v = y.reshape(-1, block)
    h = 1
    while h < block:
        p = v.reshape(-1, 2 * h)
        lo, hi = p[:, :h].copy(), p[:, h:].copy()
        p[:, :h], p[:, h:] = lo + hi, lo - hi
        h *= 2
    return y


def norm_reference_rows(x, gamma, scale, shift, row_map, rows, norm, eps, block, signs,
                        branch=None, gate=None, gate_row_map=None) -> dict:
    """Ideal prep of the sampled rows: [gated update ->] norm -> AdaLN ->
    bf16 boundary -> signs -> H -> per-row INT8 (float64 scales)."""
    idx = torch.as_tensor(rows)
    r = _f64(x[idx])
    out = {}
    if branch is not None:
        g = _f64(gate)
        gsel = g[_f64(gate_row_map[idx]).astype(int)] if gate_row_map is not None else g[None, :]
        ideal = r + gsel * _f64(branch[idx])
        out["residual_bf16"] = torch.from_numpy(ideal.astype(np.float32)).to(torch.bfloat16)
        r = _bf16_round(ideal)
    sc, sh = _f64(scale), _f64(shift)
    if row_map is not None:
        sel = _f64(row_map[idx]).astype(int)
        sc, sh = sc[sel], sh[sel]
    centered = r
    if norm == "layer":
        centered = r - r[:, :1]
        centered = centered - centered.mean(axis=1, keepdims=True)
    moment = (centered * centered).mean(axis=1, keepdims=True)
    modulated = centered / np.sqrt(moment + eps) * _f64(gamma) * (1.0 + sc) + sh
    rounded = _bf16_round(modulated)
    rotated = _fwht(rounded * _f64(signs), block)
    peak = np.abs(rotated).max(axis=1)
    scales = np.where(peak == 0, 1.0, peak / 127.0)
    codes = np.clip(np.rint(rotated / scales[:, None]), -127, 127).astype(np.int8)
    out.update(codes=codes, scales=scales, rounded_modulated=rounded, rotated=rotated)
    return out


def qk_reference_rows(dot: np.ndarray, gamma, cos, sin, eps: float, heads: int) -> np.ndarray:
    """bf16 projection -> per-head RMS over 128 -> gamma -> split-half RoPE ->
    bf16, head-major [heads, rows, 128] (float64 values)."""
    rows = dot.shape[0]
    p = _bf16_round(dot).reshape(rows, heads, 128)
    inv = 1.0 / np.sqrt((p * p).mean(axis=-1) + eps)
    u = p * inv[..., None] * _f64(gamma)
    c, s = _f64(cos), _f64(sin)
    half = c.shape[1]
    out = u.copy()
    lo, hi = u[..., :half], u[..., half:2 * half]
    out[..., :half] = lo * c[:, None, :] - hi * s[:, None, :]
    out[..., half:2 * half] = hi * c[:, None, :] + lo * s[:, None, :]
    return _bf16_round(out).transpose(1, 0, 2)


def rms_reference_rows(x_rows: np.ndarray, gamma: np.ndarray, signs: np.ndarray, block: int,
                       eps: float) -> dict:
    """Ideal folded RMS preparation of sampled rows (float64).

    The harness check of src/m5kernels/rms_quant_gemm.py:108-118: inverse RMS of
    the original rows, U = (X * gamma) D H, codes rint(U / (peak / 127)),
    scales peak / 127 * r, zero rows scale 1.
    """
    x = np.asarray(x_rows, dtype=np.float64)
    inv = 1.0 / np.sqrt((x * x).mean(axis=1) + float(eps))
    weighted = x * np.asarray(gamma, dtype=np.float64) * np.asarray(signs, dtype=np.float64)
    unscaled = weighted / np.sqrt(block) if block == 1 else _fwht(weighted, block)
    peak = np.abs(unscaled).max(axis=1)
    unit = np.where(peak == 0, 1.0, peak / 127.0)
    codes = np.clip(np.rint(unscaled / unit[:, None]), -127, 127)
    scales = np.where(peak == 0, 1.0, unit * inv)
    return {"inverse_rms": inv, "quantized": codes, "scales": scales,
            "dequantized": codes * scales[:, None],
            "normalized_rotated": unscaled * inv[:, None]}
