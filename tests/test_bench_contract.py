"""The bench's JSON line (reference arm, runnable without a GPU): one line
with the keys the harness reads, for a tiny CPU sample."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
  res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                        "--warmup", "0", "--cpu-sample-tokens", "2"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
  assert res.returncode == 0, res.stderr[-2000:]
  lines = [l for l in res.stdout.splitlines() if l.startswith("{")]
  assert len(lines) == 1
  d = json.loads(lines[0])
  for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
              "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "e2e",
              "cpu_baseline"):
    assert key in d, key
  assert d["impl"] == "reference"
  assert d["metric"] == "LatentMoE layer tokens/s" and d["unit"] == "tokens/s"
  assert d["higher_is_better"] is True and d["value"] > 0 and d["n_gpus"] == 1
  assert "workload" in d["config"] and "model" not in d["config"]
  assert d["e2e"]["value"] == d["value"]
  assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
  cb = d["cpu_baseline"]
  assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
  assert cb["sample"]
