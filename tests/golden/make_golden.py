"""Generate golden vectors by running the reference project's own CPU code.

    M5_REFERENCE_SRC=/path/to/m5-max-kernels/src python tests/golden/make_golden.py

The reference (9Tempest/m5-max-kernels) is a Python package whose CPU
references depend only on NumPy.  This script imports them from
$M5_REFERENCE_SRC (required: the reference checkout's src/ directory), runs them on small seeded inputs and writes the inputs and outputs to
tests/golden/*.npz.  The fixtures are committed; the tests never need the
reference at run time.

Reference functions exercised (file:line in the reference):
  numerics.fp8_encode / fp8_decode / quantize_reference   numerics.py:6-46
  hadamard_reference.hadamard_signs / block_hadamard_reference   hadamard_reference.py:19-68
  norm_hadamard_reference.norm_hadamard_quantize_reference   norm_hadamard_reference.py:67-94
  gated_residual_reference.gated_residual_reference   gated_residual_reference.py:21-60
  qk_rope_reference.bf16_round_reference / qk_rope_reference   qk_rope_reference.py:24-134
  rms_quant_reference.rms_quantize_reference   rms_quant_reference.py:24-89
      (written to rms_quant_vectors.npz; `--only rms` regenerates that file alone)
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _import_reference():
    src = os.environ.get("M5_REFERENCE_SRC")
    if not src:
        raise SystemExit("set M5_REFERENCE_SRC to the reference checkout's src/ directory")
    if not Path(src, "m5kernels").is_dir():
        raise SystemExit(f"reference sources not found under {src}")
    sys.path.insert(0, src)
    from m5kernels import (  # noqa: F401
        gated_residual_reference,
        hadamard_reference,
        norm_hadamard_reference,
        numerics,
        qk_rope_reference,
    )

    return numerics, hadamard_reference, norm_hadamard_reference, gated_residual_reference, qk_rope_reference


def make_rms() -> int:
    """RMS scale-folding cases (rms_quant_reference.rms_quantize_reference)."""
    _import_reference()
    from m5kernels import hadamard_reference as had
    from m5kernels import rms_quant_reference as rq

    out = {}
    cases = []

    def add(name, x, gamma, signs, block, eps=1e-5):
        x = np.asarray(x, dtype=np.float32)
        gamma = np.asarray(gamma, dtype=np.float32)
        signs = np.asarray(signs, dtype=np.int8)
        r = rq.rms_quantize_reference(x.astype(np.float64), gamma.astype(np.float64), signs, block,
                                      eps=eps)
        pre = f"rms_{name}_"
        out[pre + "x"], out[pre + "gamma"], out[pre + "signs"] = x, gamma, signs
        out[pre + "block"], out[pre + "eps"] = np.int64(block), np.float64(eps)
        for key in ("quantized", "scales", "inverse_rms", "unscaled_scales"):
            out[pre + key] = r[key]
        cases.append(name)

    rng = np.random.default_rng(2021)
    # H256 over three blocks, bf16-valued rows, signed gamma
    add("h256", bf16_value(bf16_bits(rng.standard_normal((5, 768), dtype=np.float32))),
        rng.uniform(-1.7, 1.7, 768), had.hadamard_signs(768, 61), 256)
    # no rotation, ragged K
    add("plain769", rng.standard_normal((5, 769), dtype=np.float32), rng.uniform(-1.7, 1.7, 769),
        had.hadamard_signs(769, 61), 1)
    # outlier columns under H128
    x = rng.standard_normal((4, 384), dtype=np.float32)
    x[:, ::37] *= 100
    add("outliers", x, rng.uniform(-1, 1, 384), had.hadamard_signs(384, 5), 128)
    # the peak must follow gamma and the rotation, not max |X|
    x = rng.standard_normal((3, 512), dtype=np.float32)
    x[:, 0] = 100
    gamma = rng.uniform(-1.7, 1.7, 512).astype(np.float32)
    gamma[0] = 1e-3
    gamma[1::31] *= 100
    add("weighted_peak", x, gamma, had.hadamard_signs(512, 7), 64)
    # tiny rows: epsilon dominates the RMS, codes unchanged
    add("tiny", rng.standard_normal((3, 256), dtype=np.float32) * np.float32(1e-9),
        rng.uniform(-1, 1, 256), had.hadamard_signs(256, 3), 32)
    # large epsilon
    add("eps1", rng.standard_normal((3, 512), dtype=np.float32), rng.uniform(-1, 1, 512),
        had.hadamard_signs(512, 11), 128, eps=1.0)
    # exact INT8 ties (peak 127 makes the quantizer step one)
    add("ties", [[127, 2.5, 3.5, -2.5, -3.5, 0, -127, 1.5]], np.ones(8), np.ones(8), 1)
    # a zero row among others, and an all-zero gamma
    x = rng.standard_normal((3, 256), dtype=np.float32)
    x[1] = 0
    add("zero_row", x, rng.uniform(-1, 1, 256), had.hadamard_signs(256, 13), 256)
    add("zero_gamma", np.full((3, 768), 2.0), np.zeros(768), had.hadamard_signs(768, 9), 256)
    # integer rows with unit gamma: q = rint(127 x / peak) directly
    for width in (17, 257):
        vals = np.resize(np.arange(-127, 128, dtype=np.float32), (3, width))
        add(f"int{width}", vals, np.ones(width), np.ones(width), 1)
    out["rms_cases"] = np.array(cases)

    path = HERE / "rms_quant_vectors.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size} bytes, {len(cases)} cases)")
    return 0


def bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bits (nearest even), as uint16."""
    b = np.asarray(x, dtype=np.float32).view(np.uint32)
    return ((b + np.uint32(0x7FFF) + ((b >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_value(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def main() -> int:
    if sys.argv[1:] == ["--only", "rms"]:
        return make_rms()
    make_rms()
    numerics, had, nh, gr, qk = _import_reference()
    out = {}

    # E4M3 codebook, ties, saturation and a dense sweep of float32 values.
    rng = np.random.default_rng(1234)
    sweep = np.concatenate([
        np.array([0, 2**-9, 2**-10, 1, 1.0625, 1.1875, 448, 1000, -448, -0.0, 464, 465, 2**-7], np.float32),
        (rng.standard_normal(4096) * np.exp2(rng.integers(-12, 10, 4096))).astype(np.float32),
        numerics.fp8_decode(np.arange(256, dtype=np.uint8)[np.r_[0:127, 128:255]]),
    ]).astype(np.float32)
    out["fp8_sweep_x"] = sweep
    out["fp8_sweep_code"] = numerics.fp8_encode(sweep)
    out["fp8_decode_all"] = numerics.fp8_decode(np.arange(256, dtype=np.uint8))

    # Per-token quantization, bf16 inputs (reference inputs are float32 views
    # of bf16 values), int8 / fp8 / mxint8, with zero and outlier rows.
    rng = np.random.default_rng(0)
    x = rng.standard_normal((16, 512), dtype=np.float32)
    x[3] = 0
    x[5, ::31] *= 30
    xb = bf16_bits(x)
    out["quant_x_bf16"] = xb
    xf = bf16_value(xb)
    for mode in ("int8", "fp8", "mxint8"):
        q, s = numerics.quantize_reference(xf, mode)
        out[f"quant_{mode}_q"] = q
        out[f"quant_{mode}_s"] = s
    # fp32 inputs with odd K (tail handling)
    x32 = rng.standard_normal((7, 257), dtype=np.float32)
    out["quant_x_f32_oddk"] = x32
    q, s = numerics.quantize_reference(x32, "int8")
    out["quant_oddk_int8_q"], out["quant_oddk_int8_s"] = q, s

    # Hadamard signs and rotation.
    out["signs_k512_seed17"] = had.hadamard_signs(512, 17)
    xr = rng.standard_normal((5, 512)).astype(np.float32)
    out["rot_x"] = xr
    for b in (32, 128, 256, 512):
        out[f"rot_b{b}"] = had.block_hadamard_reference(xr, b, out["signs_k512_seed17"])

    # Fused norm / modulation / rotation / INT8 (float64 ideal).
    for norm in ("rms", "layer"):
        rng = np.random.default_rng(41)
        xn = bf16_value(bf16_bits(rng.standard_normal((6, 768), dtype=np.float32)))
        gamma = rng.uniform(0.5, 1.5, 768).astype(np.float32)
        scale = rng.uniform(-0.3, 0.3, 768).astype(np.float32)
        shift = rng.uniform(-0.1, 0.1, 768).astype(np.float32)
        signs = had.hadamard_signs(768, 29)
        r = nh.norm_hadamard_quantize_reference(xn, gamma, scale, shift, 256, signs, norm=norm, eps=1e-5)
        pre = f"nhq_{norm}_"
        out[pre + "x"], out[pre + "gamma"], out[pre + "scale"], out[pre + "shift"] = xn, gamma, scale, shift
        out[pre + "signs"] = signs
        for key in ("modulated", "rotated", "quantized", "scales"):
            out[pre + key] = r[key]
    # INT8 round-half-even ties through the pipeline (block 1, zero gain).
    shift = np.array([127.0, 2.5, 3.5, -2.5, -3.5, 0.0, -127.0, 1.5])
    r = nh.norm_hadamard_quantize_reference(np.arange(24).reshape(3, 8), np.ones(8), -np.ones(8), shift, 1)
    out["ties_quantized"] = r["quantized"]
    out["ties_scales"] = r["scales"]

    # Gated residual (float64 ideal), mapped and shared gates.
    rng = np.random.default_rng(47)
    res = bf16_value(bf16_bits(rng.standard_normal((5, 131), dtype=np.float32)))
    br = bf16_value(bf16_bits(rng.standard_normal((5, 131), dtype=np.float32)))
    gt = bf16_value(bf16_bits(0.2 * rng.standard_normal((4, 131)).astype(np.float32)))
    rm = ((np.arange(5) * 3) % 4).astype(np.int32)
    out["gated_residual"], out["gated_branch"], out["gated_gate"], out["gated_row_map"] = res, br, gt, rm
    out["gated_out_table"] = gr.gated_residual_reference(res, br, gt, row_map=rm)
    out["gated_out_vec"] = gr.gated_residual_reference(res, br, gt[1])

    # BF16 rounding and Q/K RMSNorm + RoPE.
    vals = np.array([0.0, -0.0, 1.00390625, 1.01171875, -1.00390625, -1.01171875, 2.0**-134,
                     3 * 2.0**-134, -(2.0**-134), 1.00390625 + 2.0**-30])
    out["bf16_round_x"] = vals
    out["bf16_round_y"] = qk.bf16_round_reference(vals)
    rng = np.random.default_rng(103)
    proj = rng.normal(size=(5, 3, 128))
    gamma = qk.bf16_round_reference(rng.normal(size=128))
    ang = rng.uniform(-np.pi, np.pi, size=(5, 48))
    cos, sin = qk.bf16_round_reference(np.cos(ang)), qk.bf16_round_reference(np.sin(ang))
    r = qk.qk_rope_reference(proj, gamma, cos, sin, epsilon=1e-5)
    out["qk_proj"], out["qk_gamma"], out["qk_cos"], out["qk_sin"] = proj, gamma, cos, sin
    out["qk_inverse_rms"], out["qk_output"] = r["inverse_rms"], r["output"]

    path = HERE / "reference_vectors.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size} bytes, {len(out)} arrays)")
    return 0


if __name__ == "__main__":
    sys.exit(main())
