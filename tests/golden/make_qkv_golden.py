"""Golden vectors of the grouped Q/K/V post-processing from the reference's own C code.

    M5_REFERENCE_ROOT=/path/to/m5-max-kernels python tests/golden/make_qkv_golden.py

The reference's H3 integration ships an independent float64 CPU reference of
the grouped Q/K/V projection epilogue (integrations/h3/qkv_reference.h:15-36,
qvr_postprocess: BF16 projection boundary, full-head RMS, gamma before
split-half RoPE on 48 pairs, V bypassing both).  This script compiles a small
driver that includes that header from the reference checkout (nothing is
copied into this repository), runs it on seeded inputs and writes
tests/golden/qkv_vectors.npz.  The fixture is committed; tests never need the
reference or a compiler at run time.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

DRIVER = r"""
#include <stdint.h>
#include "qkv_reference.h"
/* rows x 128 projections (float64), one stream per row, shared gamma[2][128],
 * per-row cos/sin[48] (bf16 bits) -> output (float64, BF16-rounded values). */
void run(const double* proj, const int32_t* stream, const uint16_t* gamma, const uint16_t* cosine,
         const uint16_t* sine, int rows, double epsilon, double* out) {
  for (int r = 0; r < rows; ++r)
    qvr_postprocess(proj + (size_t)r * 128, (unsigned)stream[r],
                    gamma + (stream[r] == 1 ? 128 : 0), cosine + (size_t)r * 48,
                    sine + (size_t)r * 48, epsilon, out + (size_t)r * 128);
}
"""


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def main() -> int:
    env = os.environ.get("M5_REFERENCE_ROOT")
    if not env:
        raise SystemExit("set M5_REFERENCE_ROOT to the reference checkout")
    root = Path(env)
    header_dir = root / "integrations" / "h3"
    if not (header_dir / "qkv_reference.h").is_file():
        raise SystemExit(f"qkv_reference.h not found under {header_dir}")
    rng = np.random.default_rng(48)
    rows = 96
    # fp32-representable projections (the kernels' accumulator epilogue is FP32)
    proj = rng.standard_normal((rows, 128)).astype(np.float32)
    proj[0] = 0.0                      # zero row: epsilon-dominated RMS
    proj[1, ::31] *= 100.0             # outlier channels
    proj[2] *= 1e-4                    # small, epsilon-sensitive head
    stream = (np.arange(rows) % 3).astype(np.int32)  # Q, K, V interleaved
    gamma = _bf16_bits(1.0 + 0.2 * rng.standard_normal((2, 128)))
    ang = rng.uniform(-np.pi, np.pi, size=(rows, 48))
    cos_b, sin_b = _bf16_bits(np.cos(ang)), _bf16_bits(np.sin(ang))
    eps = float(np.float32(1e-5))
    out = np.zeros((rows, 128), dtype=np.float64)
    with tempfile.TemporaryDirectory() as tmp:
        src = Path(tmp, "qkv_driver.c")
        lib = Path(tmp, "libqkvref.so")
        src.write_text(DRIVER)
        subprocess.run(["gcc", "-O2", "-shared", "-fPIC", "-I", str(header_dir), str(src),
                        "-o", str(lib), "-lm"], check=True)
        so = ctypes.CDLL(str(lib))
        P = ctypes.c_void_p
        so.run.argtypes = [P, P, P, P, P, ctypes.c_int, ctypes.c_double, P]
        p64 = proj.astype(np.float64)
        so.run(p64.ctypes.data, stream.ctypes.data, gamma.ctypes.data, cos_b.ctypes.data,
               sin_b.ctypes.data, rows, eps, out.ctypes.data)
    np.savez_compressed(HERE / "qkv_vectors.npz", proj=proj, stream=stream, gamma_bits=gamma,
                        cos_bits=cos_b, sin_bits=sin_b, epsilon=np.float32(eps), output=out)
    print("wrote", HERE / "qkv_vectors.npz")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
