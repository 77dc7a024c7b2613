"""bench.py's reference arm (CPU): it must run the oracle port without mapping
this repository's own library, and report the same workload config as the GPU
arm."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_RUN = """
import runpy, sys
sys.argv = ['bench.py', '--impl', 'reference', '--steps', '1', '--warmup', '0',
            '--cpu-sample', '1', '--cpu-p50-runs', '1']
runpy.run_path('bench.py', run_name='__main__')
maps = open('/proc/self/maps').read()
print('MAPPED_PRODUCT_LIBRARY', 'libvitb200' in maps)
"""


def test_reference_arm_loads_no_product_library():
    out = subprocess.run([sys.executable, "-c", _RUN], cwd=REPO, capture_output=True, text=True,
                         timeout=600, env={**os.environ, "OMP_NUM_THREADS": "4"})
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.strip().splitlines()
    assert lines[-1] == "MAPPED_PRODUCT_LIBRARY False", lines[-1]
    rec = json.loads(lines[-2])
    assert rec["impl"] == "reference" and rec["value"] > 0
    sys.path.insert(0, REPO)
    import bench
    ours = bench.workload_config("bs256_224", 1)
    for key, val in ours.items():
        assert rec["config"][key] == val, key
    assert "cpu_sample" in rec["config"]
    assert rec["e2e"]["h2d_bytes_per_step"] == 0
