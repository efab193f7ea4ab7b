"""The debug-bounds build (libb2q_checks.so, -DB2Q_CHECKS): the kernels'
index and layout checks compiled in, standing in for a memory checker on
this pool.  tests/checks_worker.py runs GEMVs, tensor-core matmuls, a
prompt pass, persistent and graph decode steps and long-context attention
once on each library; the checks build must report its checks enabled, no
failed check and no device error, and give the regular build's outputs bit
for bit (the checks only read indices)."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = Path(__file__).resolve().parent


def _run(tmp_path, checks: bool) -> dict:
    out = tmp_path / ("checks.npz" if checks else "regular.npz")
    env = dict(os.environ, B2Q_CHECKS="1" if checks else "0")
    r = subprocess.run([sys.executable, str(HERE / "checks_worker.py"), "--out", str(out)], env=env,
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    with np.load(out) as z:
        return {k: z[k] for k in z.files}


def test_checks_build_clean_and_identical(pkg, tmp_path):
    from hf_llm_b200 import build as bld
    assert bld.lib_path(checks=True).exists(), "libb2q_checks.so is not built (build.py --checks)"
    chk = _run(tmp_path, True)
    reg = _run(tmp_path, False)
    assert int(chk["checks_enabled"]) == 1 and int(reg["checks_enabled"]) == 0
    assert int(chk["check_site"]) == 0, f"a bounds check failed at site {int(chk['check_site'])}"
    assert int(chk["device_error"]) == 0 and int(reg["device_error"]) == 0
    keys = [k for k in reg if k not in ("checks_enabled", "check_site", "device_error")]
    assert len(keys) >= 20
    for k in keys:
        assert np.isfinite(reg[k]).all(), k
        assert np.array_equal(chk[k].view(np.uint32), reg[k].view(np.uint32)), k
