"""bench.py's reference arm on the CPU: it times the oracle on host-drawn
inputs and must not load the product library (its JSON line is the driver's
reference measurement)."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

_PROBE = """
import runpy, sys
sys.argv = ['bench.py', '--impl', 'reference', '--config', 'small_fp16', '--steps', '1', '--warmup', '3',
            '--ref-sample-tokens', '16']
runpy.run_path('bench.py', run_name='__main__')
maps = open('/proc/self/maps').read()
print('LOADED', int('libsparsemoe_b200' in maps), int('sparsemoe_b200' in sys.modules))
"""


def test_reference_arm_does_not_load_the_product():
    r = subprocess.run([sys.executable, "-c", _PROBE], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = r.stdout.strip().splitlines()
    assert lines[-1] == "LOADED 0 0"
    rec = json.loads(lines[-2])
    assert rec["impl"] == "reference" and rec["unit"] == "tokens/s" and rec["value"] > 0
    assert rec["config"]["workload"] == "small_fp16" and rec["config"]["parallelism"] == "single GPU"
    assert rec["cpu_baseline"]["kind"] == "port"
    assert rec["e2e"]["h2d_bytes_per_step"] == 0
