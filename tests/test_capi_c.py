"""The C ABI driven from plain C (tests/capi_driver.c), as a cgo binding
would call it: the header compiles as C99 and the driver links against
libmimgpu.so (CPU); on a B200 the driver runs a per-op product and a whole
two-layer model and checks them bit for bit against the CPU restatement of
the reference (oracle/)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "mimir-model_b200")
ORADIR = os.path.join(ROOT, "oracle")


def _build(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    if not os.path.exists(os.path.join(LIBDIR, "libmimgpu.so")):
        pytest.fail("libmimgpu.so is missing: run mimir-model_b200/build.py")
    import oracle
    oracle.build()
    exe = str(tmp_path / "capi_driver")
    cmd = [cc, "-std=c99", "-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"), "-I", ORADIR,
           os.path.join(ROOT, "tests", "capi_driver.c"), "-o", exe,
           "-L", LIBDIR, "-lmimgpu", "-L", ORADIR, "-lmimoracle", f"-Wl,-rpath,{LIBDIR}:{ORADIR}", "-lm", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return exe


def test_c_driver_builds(tmp_path):
    assert os.path.exists(_build(tmp_path))


@pytest.mark.gpu
def test_c_driver_runs(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "capi driver ok" in r.stdout
