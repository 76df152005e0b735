"""The reference arm of bench.py (`--impl reference`), which times the CPU
restatement of the reference's path on the host cores, prints one JSON line
with the fields of the GPU arm's line plus `impl`, `cpu_baseline` and an
`e2e` that moves no bytes. Runs on the CPU (the fused elementwise chain, the
cheapest workload; the transformer takes the same code path)."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def run(*args):
    p = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args], capture_output=True,
                       text=True, timeout=600, cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, p.stdout
    return json.loads(lines[0])


def test_reference_arm_line_fields():
    d = run("--workload", "fused_elementwise", "--steps", "1", "--warmup", "0")
    assert d["impl"] == "reference"
    for k in ("metric", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling", "dtype", "data"):
        assert k in d, k
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["steps"] == 1
    assert d["ms_per_step"] > 0
    assert d["config"]["workload"].startswith("fused_elementwise")
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["unit"] == d["unit"]
    assert e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_reference_arm_decode_is_unavailable():
    d = run("--workload", "decode", "--steps", "1", "--warmup", "0")
    assert d["impl"] == "reference" and "unavailable" in d
