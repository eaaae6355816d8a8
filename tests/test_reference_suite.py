"""The reference's own tests (tests/test_correctness.py and
tests/test_correctness_extended.py of jaeeunHwang/cutlass-complex-conv),
run unmodified against this package.

The files are not copied into this repository; the test runs them from a
reference checkout beside it (``../reference/tests`` from the repository
root, or the directory named by CCV_REFERENCE_TESTS) in a child pytest
whose import path puts this package's ``complex_conv2d`` first, and skips
when no checkout is there.  Their GPU tests need CUDA and skip on a machine
without one, as in the reference; with one they run the B200 kernels.

One reference assertion is deselected by design:
``test_rejects_unsupported_options`` asserts that ``bias=True`` raises
NotImplementedError (the reference's modules.py:73-74).  This package
implements the complex bias, so that first assertion cannot hold; the same
test's other three assertions (groups, dilation, padding_mode) are checked
by tests/test_module_cpu.py::test_rejects_unsupported_options.
"""

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "cutlass-complex-conv_b200")
REF_TESTS = os.environ.get("CCV_REFERENCE_TESTS",
                           os.path.join(os.path.dirname(ROOT), "reference", "tests"))
FILES = ("test_correctness.py", "test_correctness_extended.py")
DESELECT = "not test_rejects_unsupported_options"


def _run(extra):
    env = dict(os.environ)
    env["PYTHONPATH"] = PKG_ROOT + os.pathsep + env.get("PYTHONPATH", "")
    env["PYTHONDONTWRITEBYTECODE"] = "1"
    cmd = [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "-rs",
           "--rootdir", REF_TESTS, "--import-mode=importlib", "-k", DESELECT]
    cmd += [os.path.join(REF_TESTS, f) for f in FILES] + extra
    return subprocess.run(cmd, env=env, cwd=ROOT, capture_output=True, text=True, timeout=1200)


@pytest.mark.skipif(not all(os.path.exists(os.path.join(REF_TESTS, f)) for f in FILES),
                    reason="no reference checkout beside the repository")
def test_reference_suite_passes_against_this_package():
    res = _run([])
    out = res.stdout + res.stderr
    # Without CUDA the reference's GPU tests skip themselves (as they do in
    # the reference); every test that runs must pass.
    assert res.returncode == 0, out[-4000:]
    assert "failed" not in out and "error" not in out.lower(), out[-2000:]
    # The suite imported this package, not an installed reference build.
    probe = subprocess.run(
        [sys.executable, "-c", "import complex_conv2d, os; print(os.path.abspath(complex_conv2d.__file__))"],
        env={**os.environ, "PYTHONPATH": PKG_ROOT}, capture_output=True, text=True, cwd=ROOT)
    assert probe.stdout.strip().startswith(PKG_ROOT), probe.stdout + probe.stderr
