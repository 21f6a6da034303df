"""bench.py's reference arms run on the host cores: their JSON lines keep the
contract the driver reads (one line, the keys of the GPU arm, ``impl``, a
``cpu_baseline`` that describes the run and an ``e2e`` with no copies)."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def _run(*args):
    env = dict(os.environ, H3SK_ORACLE_THREADS="4")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def _check(line, unit):
    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and line["unit"] == unit and line["value"] > 0
    assert line["cpu_baseline"]["value"] == line["value"] and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in line["config"]


@pytest.mark.parametrize("args", [("--impl", "reference", "--steps", "1", "--warmup", "0"),
                                  ("--op", "qkv", "--impl", "reference", "--steps", "1", "--tokens", "1024")])
def test_reference_arm_line(args):
    _check(_run(*args), "tokens/s")
