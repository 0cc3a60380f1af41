"""bench.py's host-side pieces without a GPU: the tensor-parallel token check
(per-sequence common prefix with one GPU's output) and the reference arm's
JSON line (a short CPU run of the oracle)."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

torch = pytest.importorskip("torch")

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402


def test_common_prefix_per_sequence():
    a = torch.tensor([[1, 2, 3, 4], [5, 6, 7, 8], [9, 9, 9, 9]])
    b = torch.tensor([[1, 2, 0, 4], [5, 6, 7, 8], [0, 9, 9, 9]])
    assert bench.common_prefix(a, b) == [2, 4, 0]
    assert bench.MIN_TP_PREFIX >= 16  # a wrong shard breaks every sequence within its first tokens


def test_reference_arm_prints_one_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "1"], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0
    assert "timed region" in line["cpu_baseline"]["sample"]
