"""bench.py's contract on a host without a GPU: the reference arm prints one
JSON line and exits 0 (rank 0), other ranks exit 0 silently; helpers of the
parity report."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _bench(*args, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=300, env=e, cwd=ROOT)


@pytest.mark.skipif(__import__("torch").cuda.is_available(), reason="checks the no-GPU reply")
def test_reference_arm_prints_one_json_line_without_a_gpu():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "1")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and "unavailable" in line


def test_reference_arm_other_ranks_exit_silently():
    r = _bench("--impl", "reference", "--steps", "1", "--warmup", "1", env={"RANK": "1", "WORLD_SIZE": "2"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_first_divergence():
    sys.path.insert(0, str(ROOT))
    import bench

    assert bench.first_divergence([1, 2, 3], [1, 2, 3]) is None
    assert bench.first_divergence([1, 2, 3], [1, 5, 3]) == 1
    assert bench.first_divergence([1, 2], [1, 2, 3]) == 2
