"""The multi-threaded CPU restatement (oracle/m5_cpu_omp.c) used as bench.py's
second CPU baseline: per-token INT8 codes and scales equal the single-threaded
restatement's, and the bf16 projection equals the epilogue over exact INT32
accumulators, for each of its inner-product kernels (AVX-512 VNNI, AVX2,
plain C) on ragged K."""

import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

CHECK = r"""
import sys, torch
sys.path.insert(0, {root!r})
from oracle import c_oracle as co
g = torch.Generator().manual_seed(3)
for (m, n, k) in [(4, 4, 16), (8, 12, 40), (64, 128, 2048), (100, 68, 1030), (12, 8, 3000)]:
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    x[1] = 0
    w = (0.02 * torch.randn(n, k, generator=g)).to(torch.bfloat16)
    wq, ws = co.quantize(w, "int8")
    out, q, s = co.omp_projection(x, wq, ws)
    q2, s2 = co.quantize(x, "int8")
    assert torch.equal(q, q2) and torch.equal(s, s2), (m, n, k)
    assert torch.equal(out, co.gemm_epilogue(co.gemm_i8_acc(q2, wq), s2, ws)), (m, n, k)
print("level", co.omp_lib().m5c_simd_level())
"""


@pytest.mark.parametrize("level", ["2", "1", "0"])
def test_omp_projection_matches_restatement(level):
    env = dict(os.environ, M5C_SIMD=level, OMP_NUM_THREADS="4")
    p = subprocess.run([sys.executable, "-c", CHECK.format(root=str(ROOT))], env=env,
                       capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-3000:]
