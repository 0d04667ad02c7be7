"""The reference arm of bench.py (`--impl reference`) runs the reference's CPU path only:
it prints one JSON line with the contract's keys and maps no part of this repository's
CUDA library into its process."""

from __future__ import annotations

import json
import subprocess
import sys

from conftest import ROOT

_PROBE = """
import json, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "2", "--warmup", "1"]
sys.path.insert(0, {root!r})
import bench
bench.main()
maps = open("/proc/self/maps").read()
print(json.dumps({{"fusion_so_mapped": "libfusion_b200" in maps,
                   "fusion_modules": sorted(m for m in sys.modules if m.startswith("fusion_b200"))}}))
"""


def test_reference_arm_loads_no_fusion_library():
    r = subprocess.run([sys.executable, "-c", _PROBE.format(root=str(ROOT))], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    line, probe = json.loads(lines[-2]), json.loads(lines[-1])
    assert line["impl"] == "reference"
    for k in ("metric", "value", "unit", "config", "cpu_baseline", "e2e", "higher_is_better"):
        assert k in line, k
    assert line["value"] > 0 and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0
    assert not probe["fusion_so_mapped"]
    assert probe["fusion_modules"] == []
