"""The C host program in tests/c (the engine's use of the C ABI) builds
against include/*.h and libsf37kv.so with a plain C compiler; on a GPU it
runs and checks itself."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c", "dropin_host.c")
LIBDIR = os.path.join(ROOT, "sf37_b200")


def _build(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if not cc:
        pytest.skip("no C compiler")
    exe = os.path.join(str(tmp_path), "dropin_host")
    r = subprocess.run([cc, "-std=c11", "-O2", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), SRC,
                        "-L", LIBDIR, "-lsf37kv", "-Wl,-rpath," + LIBDIR, "-lm", "-o", exe],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_c_host_builds(tmp_path):
    _build(tmp_path)


@pytest.mark.gpu
def test_c_host_runs(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("OK")
