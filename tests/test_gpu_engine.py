"""The cuda-b200 backends through the harness: every smoke case must pass the
reference-style gates (implementation error, online path, transform checks)
and be timed."""

import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine():
    from m5kernels_b200 import engine as e

    return e


def test_smoke_suite_passes_and_is_timed(engine):
    from m5kernels_b200 import workloads

    for c in workloads.load("smoke")["cases"]:
        backend = engine.BACKENDS[c["op"]][0]
        if c["op"] == "gemm" and "hadamard" in c:
            backend = "cuda-b200-hadamard"
        r = engine.run_case(c, backend, "int8", warmup=1, repeat=3)
        assert r["status"] == "ok", (c["id"], r.get("reason"), r.get("implementation_error"))
        assert r["timing"]["median_ms"] > 0 and r["effective_tops"] > 0


@pytest.mark.parametrize("precision", ["int8", "fp8"])
def test_gemm_case_fp8_and_outliers(engine, precision):
    c = dict(id="t", op="gemm", m=300, n=520, k=1024, weight_std=0.02)
    r = engine.run_case(c, "cuda-b200", precision, distribution="outliers", warmup=1, repeat=2)
    assert r["status"] == "ok", r.get("reason")
