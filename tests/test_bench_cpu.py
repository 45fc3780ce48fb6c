"""bench.py's reference arm on CPU: the JSON line the driver reads (the
reference's own compiled core timed on the host cores), and the other ranks of
a multi-process launch exiting quietly."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
LIBREF = REPO / "oracle" / "_ref" / "liboracle.so"


def _run(tmp_path, **env):
    cmd = [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0",
           "--workdir", str(tmp_path)]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=dict(os.environ, **env))


@pytest.mark.skipif(not LIBREF.exists(), reason="reference core not built (oracle/Makefile)")
def test_reference_arm_prints_the_contract_line(tmp_path):
    r = _run(tmp_path)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [line for line in r.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["unit"] == "chunks/s" and d["value"] > 0 and d["steps"] == 1
    assert d["config"]["global_batch"] == 4096
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_without_output(tmp_path):
    r = _run(tmp_path, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
