"""bench.py's reference arm and its JSON contract, on the CPU.

`bench.py --impl reference` times the reference's CPU path (the oracle port
of quantize_reference + the decoded GEMM) on the host cores and prints one
JSON line with the headline metric, unit and config, a cpu_baseline object
and an e2e object with zero copy bytes.  Under torchrun only rank 0 works and
prints; the other ranks exit 0 without output.
"""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(extra_env=None):
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    env.update(extra_env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "3"], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    p = _run()
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    base = json.loads((ROOT / "BASELINE.json").read_text())
    assert d["impl"] == "reference"
    assert d["metric"] == base["metric"]
    assert d["unit"] == "TOPS" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["scaling"] == "strong" and d["n_gpus"] == 1 and d["steps"] == 1
    assert d["config"]["workload"].startswith("ffn_down")
    # the same config dict as the CUDA arm's line at this GPU count
    sys.path.insert(0, str(ROOT))
    import bench

    assert d["config"] == bench._config(1)
    assert d["config"]["global_M"] == 4096 and d["rows_per_step"] == 4096  # the full job per step
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert "OMP_NUM_THREADS" in cb["threads"] and "OPENBLAS_NUM_THREADS" in cb["threads"]
    assert d["e2e"] == {"value": d["value"], "unit": "TOPS", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_nonzero_rank_exits_quietly():
    p = _run({"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [l for l in p.stdout.splitlines() if l.startswith("{")]
