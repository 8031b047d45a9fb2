"""The reference's own test suite, unmodified, against this package.

The reference's ``src/tests/test_*.py`` (28 items: test_siso.py,
test_mimo.py, test_trapezoidal.py, test_full_fused.py) import
``src.kernels.*`` and ``src.models.*``.  Here they run in a child pytest
with this package's directory as the only ``src`` on the path, so every
kernel function and the ``Mamba3Decoder`` they call are this package's
CUDA-backed ones.  The files come byte for byte from the copy that
``oracle/stage_reference.py`` staged under ``baseline/_ref`` (checked
against its sha256 manifest) and are copied into an empty temporary
directory, away from the reference's own ``src`` package.  A conftest
written beside them checks which ``src`` was imported and reports whether
the CUDA library was mapped into the child process.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

import pytest

from conftest import PKG
from oracle.stage_reference import DEFAULT_OUT, verify

pytestmark = pytest.mark.gpu
EXPECTED_ITEMS = 28

CHILD_CONFTEST = '''
import os

import src

PKG = os.environ["M3_PACKAGE_DIR"]
assert os.path.dirname(os.path.dirname(os.path.abspath(src.__file__))) == PKG, src.__file__


def pytest_sessionfinish(session, exitstatus):
    with open("/proc/self/maps") as f:
        loaded = "libmamba3_b200.so" in f.read()
    print(f"\\nM3_NATIVE_LOADED={loaded}")
'''


def test_reference_suite_passes_against_this_package(tmp_path):
    why = verify(DEFAULT_OUT)
    if why:
        pytest.skip(why)
    src_tests = os.path.join(DEFAULT_OUT, "src", "tests")
    names = sorted(n for n in os.listdir(src_tests) if n.startswith("test_") and n.endswith(".py"))
    assert names == ["test_full_fused.py", "test_mimo.py", "test_siso.py", "test_trapezoidal.py"]
    for name in names:
        shutil.copyfile(os.path.join(src_tests, name), tmp_path / name)
    (tmp_path / "conftest.py").write_text(CHILD_CONFTEST)
    env = dict(os.environ, PYTHONPATH=PKG, M3_PACKAGE_DIR=PKG, PYTHONDONTWRITEBYTECODE="1")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-rA", "-p", "no:cacheprovider",
                        "--rootdir", str(tmp_path), str(tmp_path)],
                       cwd=tmp_path, env=env, capture_output=True, text=True, timeout=900)
    tail = r.stdout[-4000:] + r.stderr[-2000:]
    assert r.returncode == 0, tail
    assert f"{EXPECTED_ITEMS} passed" in r.stdout, tail
    assert "M3_NATIVE_LOADED=True" in r.stdout, tail
