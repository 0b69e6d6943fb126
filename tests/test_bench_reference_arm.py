"""bench.py's reference arm (the reference's own CPU layer) prints one JSON line
with the contract's keys: impl, metric/unit matching our arm, cpu_baseline and
an e2e block with no host<->device bytes.  Runs on CPU at a small token count."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_json_line():
    if not (ROOT / "baseline" / "_ref" / "cuda_qwen3_vl").exists():
        pytest.skip("reference package not installed beside the repository")
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                          "--warmup", "1", "--tokens", "256"], cwd=ROOT, capture_output=True,
                         text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "moe_layer_prefill_tokens_per_s" and line["unit"] == "tokens/s"
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] in ("reference", "port")
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
