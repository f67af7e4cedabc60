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


@pytest.mark.parametrize("backend", ["cuda-b200-rms-folded", "cuda-b200-rms-direct"])
@pytest.mark.parametrize("distribution", ["normal", "outliers", "zeros"])
@pytest.mark.parametrize("block,gamma,sign_seed", [(1, "identity", None), (256, "random", 3)])
def test_rms_quant_gemm_backends(engine, backend, distribution, block, gamma, sign_seed):
    c = dict(id="t.rms", op="rms_quant_gemm", m=300, n=384, k=1280,
             rms_quant=dict(block_size=block, gamma=gamma, sign_seed=sign_seed))
    r = engine.run_case(c, backend, "int8", distribution=distribution, warmup=1, repeat=2)
    assert r["status"] == "ok", (r.get("reason"), r.get("activation_implementation_error"))
    assert r["transform_pass"] and r["activation_max_code_difference"] <= 1
    assert set(r["stages"]) == {"activation_prepare", "online_activation_plus_gemm",
                                "offline_weight_prepare"}


def test_rms_folded_and_direct_share_inputs(engine):
    c = dict(id="t.rms", op="rms_quant_gemm", m=256, n=256, k=768,
             rms_quant=dict(block_size=256, gamma="random", sign_seed=1))
    a = engine.run_case(c, "cuda-b200-rms-folded", "int8", warmup=1, repeat=2)
    b = engine.run_case(c, "cuda-b200-rms-direct", "int8", warmup=1, repeat=2)
    assert a["status"] == b["status"] == "ok"
    assert a["gamma_sha256"] == b["gamma_sha256"]


@pytest.mark.parametrize("op,backends", [
    ("norm_hadamard_gemm", ("cuda-b200-norm-fused", "cuda-b200-norm-staged")),
    ("gated_norm_hadamard_gemm", ("cuda-b200-residual-fused", "cuda-b200-residual-separate")),
    ("qk_rope", ("cuda-b200-qk-fused", "cuda-b200-qk-staged")),
])
def test_staged_and_fused_backends_agree_exactly(engine, op, backends):
    """Each fused backend has a staged comparator with bit-identical results."""
    c = dict(id="t.pair", op=op, m=520, n=384, k=2048,
             fusion=dict(norm="layer", epsilon=1e-6, block_size=128, samples=2))
    results = [engine.run_case(c, b, "int8", warmup=1, repeat=2) for b in backends]
    for r in results:
        assert r["status"] == "ok", (r["backend"], r.get("reason"))
        assert r["paired_path_exact"] is True
    assert results[0]["compute_path"] != results[1]["compute_path"]


def test_tune_selects_a_schedule_and_passes_the_holdout(tmp_path):
    """The tune twin: eight schedules of the C1 GEMM, the fastest correct one
    re-run on a fresh seed (reference: src/m5kernels/cli.py:66-151)."""
    import json

    from m5kernels_b200 import cli

    out = tmp_path / "tune.json"
    rc = cli.main(["tune", "--suite", "baseline", "--filter", "c1.", "--warmup", "1",
                   "--repeat", "3", "--out", str(out)])
    doc = json.loads(out.read_text())
    assert rc == 0
    assert len(doc["results"]) == len(cli.SCHEDULES)
    assert all(r["status"] == "ok" for r in doc["results"])
    (sel,) = doc["selections"]
    assert sel["holdout"]["seed"] == 18 and sel["holdout"]["status"] == "ok"
    assert sel["holdout"]["schedule"] == sel["schedule"]
