"""bench.py's reference arm (the oracle on the host's cores) prints the one
JSON line the contract asks for, with no GPU, and never loads the product
library."""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.timeout(600)
def test_reference_arm_prints_its_line():
    env = dict(os.environ)
    env.setdefault("NEEDLE_BENCH_CACHE", os.environ.get("NEEDLE_TEST_CACHE", "/tmp/needle_b200_test_cache"))
    # run the arm in a process that then reports whether the product
    # library was ever mapped into it (the arm must not load it)
    code = ("import runpy, sys\n"
            f"sys.argv = [{os.path.join(ROOT, 'bench.py')!r}, '--impl', 'reference', '--steps', '1', '--warmup', '1']\n"
            "runpy.run_path(sys.argv[0], run_name='__main__')\n"
            "print('product mapped:', 'libneedle3' in open('/proc/self/maps').read())\n")
    out = subprocess.check_output([sys.executable, "-c", code], env=env, text=True, cwd=ROOT)
    assert "product mapped: False" in out
    lines = [ln for ln in out.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["higher_is_better"] is True and d["unit"] == "tok/s"
    assert d["value"] > 0 and d["steps"] == 1 and d["warmup"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "agent_decode"
