"""The bounds-checked build (``-DRO_BOUNDS_CHECK``, module ``_C_checked``):
the kernel oracle tests pass under it without one failed index check, and a
failed check is recorded (site and source line) with the guarded store
skipped instead of a fault."""
import glob
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "rational_optimizer_b200")


def _env(tmp_path):
    if not glob.glob(os.path.join(PKG, "_C_checked*.so")):
        pytest.fail("the bounds-checked build is missing: "
                    "RO_BOUNDS_CHECK=1 python setup.py build_ext --inplace --build-temp build/checked")
    return dict(os.environ, RO_CHECKED="1", RO_CHECKED_REPORT=str(tmp_path / "faults.json"),
                PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))


def test_kernel_oracles_pass_under_the_checked_build(tmp_path):
    env = _env(tmp_path)
    run = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                          "tests/test_kernels_gpu.py", "tests/test_optim_gpu.py"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert run.returncode == 0, run.stdout[-3000:] + run.stderr[-3000:]
    report = json.loads((tmp_path / "faults.json").read_text())
    assert report["checked"] and report["module"].split(os.sep)[-1].startswith("_C_checked")
    assert report["faults"] == {"grain": 0, "nn_ops": 0, "optim": 0}, report


def test_a_failed_check_is_recorded_and_the_access_skipped(tmp_path):
    env = _env(tmp_path)
    code = (
        "import json, torch\n"
        "from rational_optimizer_b200 import _ext\n"
        "C = _ext.ext()\n"
        "buf = torch.zeros(17, device='cuda')\n"
        "C.bounds_selftest(buf, 16)\n"
        "ok = C.bounds_faults()\n"
        "C.bounds_selftest(buf[:16], 16)\n"  # one past the end of a 16-element view
        "bad = C.bounds_faults()\n"
        "again = C.bounds_faults()\n"
        "print(json.dumps({'ok': ok, 'bad': bad, 'again': again, 'buf': buf.tolist()}))\n")
    run = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=300)
    assert run.returncode == 0, run.stderr[-3000:]
    out = json.loads(run.stdout.strip().splitlines()[-1])
    assert out["ok"] == {"grain": 0, "nn_ops": 0, "optim": 0}
    word = out["bad"]["nn_ops"]
    assert word >> 32 == 99 and (word & 0xFFFFFFFF) > 0  # site 99 at a source line
    assert out["bad"]["grain"] == out["bad"]["optim"] == 0
    assert out["again"]["nn_ops"] == 0  # reading clears the word
    assert out["buf"][16] == 1.0  # the in-bounds call wrote its element ...
    assert sum(out["buf"][:16]) == 0.0  # ... the checked-out call wrote nothing
