"""The index-checked build (libmoteopt_checked.so, -DMOTE_OPT_CHECKS) on a workload that reaches every kernel:
no index check fails, no status bit is raised, and the outputs equal the release library's bit for bit (the checks
only count, they change no arithmetic). The stand-in for a memory checker on GPUs where none runs."""

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def _run(lib: Path, out: Path) -> dict:
    env = dict(os.environ, MOTEOPT_LIB=str(lib))
    r = subprocess.run([sys.executable, str(ROOT / "tests" / "checked_workload.py"), str(out)], env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = dict(ln.split(None, 1) for ln in r.stdout.strip().splitlines()[-2:])
    return {"status": int(lines["status"]), "checks": int(lines["checks"])}


def test_checked_build_finds_no_bad_index_and_matches_the_release_build(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    checked = ROOT / "mote_b200" / "libmoteopt_checked.so"
    release = ROOT / "mote_b200" / "libmoteopt.so"
    assert checked.exists(), "build it with `python -m mote_b200.build --checked` (__graft_entry__.build does)"
    a = _run(checked, tmp_path / "checked.npz")
    b = _run(release, tmp_path / "release.npz")
    assert a["checks"] == 0 and b["checks"] == 0
    assert a["status"] & 3 == 0 and b["status"] & 3 == 0
    x, y = np.load(tmp_path / "checked.npz"), np.load(tmp_path / "release.npz")
    assert sorted(x.files) == sorted(y.files)
    for k in x.files:   # bit for bit (NaN-safe): compare the bytes
        assert np.array_equal(np.ascontiguousarray(x[k]).reshape(-1).view(np.uint8),
                              np.ascontiguousarray(y[k]).reshape(-1).view(np.uint8)), k
