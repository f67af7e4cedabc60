"""Versioned workload manifests for the cuda-b200 backend (schema v1).

Same case schema as the reference's src/m5kernels/workloads.py:9-37: each
case has a unique `id`, an `op` and positive integer shape fields; optional
per-op sub-configs (`hadamard`, `fusion`, `rope_half`, `epsilon`).  The
built-in suite "baseline" holds the five BASELINE configurations of this
build (seeded synthetic data; no dataset is involved).
"""

from __future__ import annotations

import json
from pathlib import Path

FIELDS = {
    "gemm": ("m", "n", "k"),
    "norm_hadamard_gemm": ("m", "n", "k"),
    "gated_norm_hadamard_gemm": ("m", "n", "k"),
    "qk_rope": ("m", "n", "k"),
    "rms_quant_gemm": ("m", "n", "k"),
}


def validate(c: dict) -> dict:
    if not isinstance(c.get("id"), str) or not c["id"]:
        raise ValueError("nonempty id required")
    if c.get("op") not in FIELDS:
        raise ValueError(f"unknown op {c.get('op')!r}")
    for f in FIELDS[c["op"]]:
        if type(c.get(f)) is not int or c[f] < 1:
            raise ValueError(f"{f} must be a positive integer")
    return c


def _baseline_cases():
    cases = [dict(id="c1.w8a8.m512", op="gemm", m=512, n=2048, k=2048, weight_std=0.02,
                  component="config1_cpu_reference_case")]
    for m in (4096, 9914):
        for name, k, n in (("q", 4096, 4096), ("ffn_up", 4096, 16384), ("ffn_down", 16384, 4096)):
            cases.append(dict(id=f"c2.{name}.m{m}", op="gemm", m=m, n=n, k=k, weight_std=0.02,
                              component=name))
    cases.append(dict(id="c3.ffn_down.h128.m4096", op="gemm", m=4096, n=4096, k=16384,
                      weight_std=0.02, hadamard=dict(block_size=128), component="ffn_down"))
    cases.append(dict(id="c4.gated_prep_q.m4096", op="gated_norm_hadamard_gemm", m=4096, n=4096,
                      k=4096, fusion=dict(norm="layer", epsilon=1e-6, block_size=128,
                                          samples=2, affine=False)))
    cases.append(dict(id="c5.qk_rope.m9914", op="qk_rope", m=9914, n=4096, k=4096, rope_half=64,
                      theta=10000.0, gamma_std=0.02))
    return cases


def _rms_cases():
    # the reference's rms-quant manifest shapes: Q-sized GEMM, zero-shift RMS prep
    cases = []
    for m in (4096, 9914):
        for name, block, gamma in (("plain", 1, "identity"), ("weighted", 1, "random"),
                                   ("weighted_h256", 256, "random")):
            cases.append(dict(id=f"rms.{name}.m{m}", op="rms_quant_gemm", m=m, n=7168, k=5376,
                              rms_quant=dict(block_size=block, gamma=gamma, threads=256,
                                             epsilon=1e-5)))
    return cases


SUITES = {
    "baseline": {"schema_version": 1, "cases": _baseline_cases()},
    "smoke": {"schema_version": 1, "cases": [
        dict(id="smoke.gemm", op="gemm", m=130, n=384, k=512),
        dict(id="smoke.hadamard", op="gemm", m=65, n=256, k=1024, hadamard=dict(block_size=128)),
        dict(id="smoke.gated", op="gated_norm_hadamard_gemm", m=96, n=256, k=512,
             fusion=dict(norm="layer", epsilon=1e-6, block_size=128, samples=2)),
        dict(id="smoke.norm", op="norm_hadamard_gemm", m=64, n=256, k=768,
             fusion=dict(norm="rms", block_size=256)),
        dict(id="smoke.qk", op="qk_rope", m=77, n=256, k=512, rope_half=48),
        dict(id="smoke.rms", op="rms_quant_gemm", m=70, n=256, k=768,
             rms_quant=dict(block_size=256, gamma="random", sign_seed=5)),
    ]},
    "rms_quant": {"schema_version": 1, "cases": _rms_cases()},
}


def load(name: str) -> dict:
    """Load a built-in suite by name, or a JSON manifest file by path."""
    if name in SUITES:
        data = json.loads(json.dumps(SUITES[name]))
    else:
        data = json.loads(Path(name).read_text())
    cases = [validate(c) for c in data["cases"]]
    if len({c["id"] for c in cases}) != len(cases):
        raise ValueError("duplicate case id")
    return data
