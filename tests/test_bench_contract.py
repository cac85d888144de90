"""bench.py's reference arm runs on the host alone: it must print one JSON
line with the keys and meanings the benchmark contract asks for, describe
the same workload (``config``) as our arm, and never load this library."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

# Runs bench.py's reference arm in-process, then reports whether the product
# package was imported or its shared library mapped into the process.
_PROBE = r"""
import json, runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "3"]
runpy.run_path("bench.py", run_name="__main__")
maps = open("/proc/self/maps").read()
print(json.dumps({"probe": {"phantom_moe_imported": any(m.startswith("phantom_moe") for m in sys.modules),
                            "libphmoe_mapped": "libphmoe" in maps}}))
"""


def test_reference_arm_prints_the_contract_line():
    proc = subprocess.run([sys.executable, "-c", _PROBE], cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.strip()]
    assert len(lines) == 2, proc.stdout
    d, probe = json.loads(lines[0]), json.loads(lines[1])["probe"]
    assert not probe["phantom_moe_imported"] and not probe["libphmoe_mapped"], probe
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 3
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    # the same workload description our arm prints with default flags at N = 1
    sys.path.insert(0, str(ROOT))
    import bench
    args = bench.build_parser().parse_args([])
    assert d["config"] == bench.bench_config(1, args.tokens, args)
