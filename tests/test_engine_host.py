"""Host-side harness logic that needs no GPU: manifests, statuses, result files,
and the rule that an incorrect implementation is never timed (fault injected on
the host by a corrupted prepare, as the reference's tests do with monkeypatch)."""

import json

import numpy as np
import pytest
import torch

from m5kernels_b200 import engine, workloads


def test_baseline_suite_holds_the_five_configs():
    data = workloads.load("baseline")
    ids = [c["id"] for c in data["cases"]]
    assert data["schema_version"] == 1
    assert "c1.w8a8.m512" in ids and "c2.ffn_down.m4096" in ids and "c2.ffn_down.m9914" in ids
    assert "c3.ffn_down.h128.m4096" in ids and "c4.gated_prep_q.m4096" in ids
    assert "c5.qk_rope.m9914" in ids
    down = next(c for c in data["cases"] if c["id"] == "c2.ffn_down.m4096")
    assert (down["m"], down["k"], down["n"]) == (4096, 16384, 4096)


def test_manifest_validation(tmp_path):
    with pytest.raises(ValueError):
        workloads.validate(dict(id="bad", op="gemm", m=-1, n=1, k=1))
    with pytest.raises(ValueError):
        workloads.validate(dict(id="", op="gemm", m=1, n=1, k=1))
    p = tmp_path / "dup.json"
    p.write_text(json.dumps({"schema_version": 1, "cases": [dict(id="a", op="gemm", m=1, n=1, k=1)] * 2}))
    with pytest.raises(ValueError, match="duplicate"):
        workloads.load(str(p))


def test_unknown_backend_is_unsupported_not_error():
    r = engine.run_case(dict(id="x", op="gemm", m=8, n=8, k=32), "mpp", "int8")
    assert r["status"] == "unsupported" and "timing" not in r


def test_unknown_op_is_unsupported():
    r = engine.run_case(dict(id="x", op="attention", m=8, n=8, k=32), "cuda-b200", "int8")
    assert r["status"] == "unsupported"


def test_incorrect_result_is_never_timed(monkeypatch):
    """A corrupted kernel output must give status 'incorrect' and no timing."""
    expected = np.ones((4, 4))

    def corrupted_prepare(c, backend, precision, seed, distribution, tile):
        y = torch.full((4, 4), 2.0)
        stages = {"online_activation_plus_gemm": lambda: y}
        return (lambda: y), (lambda t: t.double().numpy()), expected, expected, stages, \
            dict(mac_operations=128)

    monkeypatch.setitem(engine.PREPARE, "gemm", corrupted_prepare)
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda: (1 << 40, 1 << 40))
    monkeypatch.setattr(torch.cuda, "synchronize", lambda: None)
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: None)
    monkeypatch.setattr(engine._lib, "device_status", lambda clear=False: 0)
    timed_calls = []
    monkeypatch.setattr(engine, "timed", lambda *a, **k: timed_calls.append(1))
    r = engine.run_case(dict(id="x", op="gemm", m=4, n=4, k=32), "cuda-b200", "int8")
    assert r["status"] == "incorrect"
    assert r["implementation_error"]["relative_l2"] > 0.5
    assert "timing" not in r and not timed_calls


def test_device_status_word_marks_case_incorrect(monkeypatch):
    """A bounded device wait that gave up (status word != 0) fails the case."""
    expected = np.ones((4, 4))

    def prepare(c, backend, precision, seed, distribution, tile):
        y = torch.ones(4, 4)
        return (lambda: y), (lambda t: t.double().numpy()), expected, expected, \
            {"online_activation_plus_gemm": lambda: y}, dict(mac_operations=128)

    monkeypatch.setitem(engine.PREPARE, "gemm", prepare)
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "mem_get_info", lambda: (1 << 40, 1 << 40))
    monkeypatch.setattr(torch.cuda, "synchronize", lambda: None)
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: None)
    monkeypatch.setattr(engine._lib, "device_status", lambda clear=False: 0x2)
    monkeypatch.setattr(engine, "timed", lambda *a, **k: pytest.fail("must not time"))
    r = engine.run_case(dict(id="x", op="gemm", m=4, n=4, k=32), "cuda-b200", "int8")
    assert r["status"] == "incorrect" and r["device_status"] == 2


def test_write_result_is_exclusive(tmp_path):
    p = tmp_path / "r.json"
    engine.write_result(p, {"a": 1})
    with pytest.raises(FileExistsError):
        engine.write_result(p, {"a": 2})
    assert json.loads(p.read_text()) == {"a": 1}


def test_cli_shapes_and_doctor_without_gpu(capsys):
    from m5kernels_b200 import cli

    assert cli.main(["shapes", "--suite", "baseline"]) == 0
    out = capsys.readouterr().out
    assert "c2.ffn_down.m4096" in out
    rc = cli.main(["doctor"])
    assert rc == (0 if torch.cuda.is_available() else 1)


def test_cli_tune_records_every_schedule(tmp_path, capsys):
    """Without a device every schedule's run is recorded as an error and no
    selection is made (exit 1); with no matching GEMM case tune refuses."""
    from m5kernels_b200 import cli

    if torch.cuda.is_available():
        pytest.skip("host-only behaviour")
    out = tmp_path / "tune.json"
    assert cli.main(["tune", "--suite", "baseline", "--filter", "c1.", "--out", str(out)]) == 1
    doc = json.loads(out.read_text())
    assert [tuple(r["schedule"].values()) for r in doc["results"]] == cli.SCHEDULES
    assert all(r["status"] == "error" for r in doc["results"]) and doc["selections"] == []
    with pytest.raises(FileExistsError):
        cli.main(["tune", "--suite", "baseline", "--filter", "c1.", "--out", str(out)])
    with pytest.raises(ValueError, match="no GEMM cases"):
        cli.main(["tune", "--suite", "baseline", "--filter", "c4."])


def test_rms_case_semantics_are_validated_before_any_device_work():
    from m5kernels_b200 import engine

    base = dict(id="r", op="rms_quant_gemm", m=8, n=8, k=512)
    ok = engine.validate_rms_config(base, "cuda-b200-rms-folded", "int8", "normal")
    assert ok["block_size"] == 1 and ok["gamma"] == "identity" and ok["threads"] == 256
    for bad, err in [
        (dict(base, shift=1), NotImplementedError),
        (dict(base, rms_quant=dict(block_size=128)), NotImplementedError),
        (dict(base, rms_quant=dict(gamma="learned")), NotImplementedError),
        (dict(base, rms_quant=dict(threads=64)), NotImplementedError),
        (dict(base, rms_quant=dict(epsilon=0)), ValueError),
        (dict(base, rms_quant=dict(epsilon=1e-300)), ValueError),
        (dict(base, rms_quant=dict(sign_seed=-1)), ValueError),
        (dict(base, rms_quant=dict(norm="layer")), NotImplementedError),
        (dict(base, k=300, rms_quant=dict(block_size=256)), NotImplementedError),
    ]:
        with pytest.raises(err):
            engine.validate_rms_config(bad, "cuda-b200-rms-folded", "int8", "normal")
    with pytest.raises(NotImplementedError):
        engine.validate_rms_config(base, "cuda-b200-rms-folded", "fp8", "normal")
    with pytest.raises(NotImplementedError):
        engine.validate_rms_config(base, "cuda-b200", "int8", "normal")


def test_rms_suite_mirrors_the_reference_manifest():
    from m5kernels_b200 import workloads

    cases = workloads.load("rms_quant")["cases"]
    assert [c["id"] for c in cases] == [
        "rms.plain.m4096", "rms.weighted.m4096", "rms.weighted_h256.m4096",
        "rms.plain.m9914", "rms.weighted.m9914", "rms.weighted_h256.m9914"]
    assert all((c["n"], c["k"]) == (7168, 5376) for c in cases)
