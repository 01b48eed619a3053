"""CPU: the benchmark's byte accounting and its reference arm's output line.

The bench credits each attention call with the algorithmic bytes of the decode/verify step
(K and V history, page-table entries, Q in and O out) and nothing else; the reference arm
times the reference's eager attention formula on the host and prints one JSON line with the
same metric and workload as the GPU arm.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("T", [16, 2048, 8192])
@pytest.mark.parametrize("q", [1, 5])
def test_attention_bytes_per_call(T, q):
    """1024.25 B per key (bf16 K and V of 2 KV heads x 128 dims, 4 B of page table per 16
    keys) and 776.25 B with E4M3 V (1 B codes + a 4 B scale per token and head), plus
    6144 B per query position (12 heads x 128 dims of bf16 Q in and O out)."""
    import bench

    assert bench.attn_bytes(T, q, False) == 1024.25 * T + 6144 * q
    assert bench.attn_bytes(T, q, True) == 776.25 * T + 6144 * q


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    line = json.loads(lines[-1])
    assert line["impl"] == "reference"
    assert line["unit"] == "GB/s" and line["value"] > 0 and line["higher_is_better"] is True
    assert "unavailable" not in line
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["e2e"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] in ("port", "reference") and line["cpu_baseline"]["cores"] >= 1
    assert "workload" in line["config"]
