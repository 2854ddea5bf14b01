"""This library against the reference itself on the GPU: COMP's own Triton kernels (installed under baseline/_ref by
baseline/install_ref.sh, JIT-compiled for the B200) and this library's kernels on the same seeded inputs at BASELINE's
full sizes (configs 0, 1, 3 and 4): the quantized activation bytes and every int32 block dot are identical, and Y is
within KURN's 1e-5 relative-error rule of the reference's Y (tests/komp_worker.py)."""

import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
TOL = 1e-5  # KURN's rule (src/komp/verify.py:28)


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "komp", "host.py")),
                    reason="the reference is not installed under baseline/_ref (baseline/install_ref.sh)")
def test_full_size_layers_match_comps_own_kernels(tmp_path):
    env = {k: v for k, v in os.environ.items() if k != "TRITON_INTERPRET"}
    env["KOMP_PATCHES"] = os.path.join(REF, "patches")
    env["KOMP_CACHE"] = str(tmp_path / "komp_cache")
    env["PYTHONPATH"] = REF + os.pathsep + env.get("PYTHONPATH", "")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "komp_worker.py")], capture_output=True,
                       text=True, timeout=900, env=env, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    rows = [json.loads(line) for line in r.stdout.splitlines() if line.startswith("{")]
    assert len(rows) == 8, r.stdout[-3000:]
    for row in rows:
        assert row["quant_bytes_equal"], row
        assert row["int32_block_dots_equal"], row
        assert row["relerr_separate"] <= TOL and row["relerr_fused"] <= TOL, row
