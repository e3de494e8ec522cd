"""bench.py's reference arm on the CPU: the reference's own CPU path
(oracle/_ref, compiled from its sources) on a small sample prints one JSON
line with the fields the measurement contract names, and a rank other than
0 prints nothing."""
import glob
import json
import os
import subprocess
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _ref_built():
    return bool(glob.glob(os.path.join(ROOT, "oracle", "_ref", "cascade_ref*.so")))


def _run(env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    return subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                           "--cpu-blocks", "128"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


@pytest.mark.skipif(not _ref_built(), reason="oracle/_ref not built")
def test_reference_arm_line():
    out = _run()
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
              "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert k in line, k
    assert line["unit"] == "GB/s" and line["value"] > 0 and line["higher_is_better"] is True
    assert abs(line["value_gibs"] - line["value"] * 1e9 / 2**30) < 0.01
    assert line["steps"] == 1 and line["n_gpus"] == 1 and line["vs_baseline"] is None
    assert "workload" in line["config"]
    cb = line["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["value"] == line["value"] and cb["cores"] >= 1 and "128" in cb["sample"]
    assert isinstance(cb["cpu_model"], str) and isinstance(cb["sha_ni"], bool)
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    # ms_per_step is the timed put + get of the step: value x time = the
    # step's logical bytes (every block put + every unique block read back)
    from cascade_cpp import workloads as W
    src, _ = W.dedup_mix(128, 2, 0.25, 77)
    logical = (128 + len(np.unique(src))) * 917504
    assert abs(line["value"] * 1e9 * line["ms_per_step"] / 1e3 - logical) <= 0.01 * logical


def test_reference_arm_other_ranks_print_nothing():
    out = _run({"RANK": "1", "WORLD_SIZE": "2"})
    assert out.returncode == 0
    assert out.stdout.strip() == ""
