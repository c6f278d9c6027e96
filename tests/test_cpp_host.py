"""The C++ host mirror (include/qw/mlxcel.hpp): its tests (tests/cpp/
test_mlxcel_host.cpp, written like the reference's ffi_tests.rs) build here
without a GPU and run on one."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tests", "cpp", "_build", "test_mlxcel_host")


def _build():
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "qw_b200", "csrc")], check=True)
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp")], check=True)


def test_cpp_host_mirror_builds():
    _build()
    assert os.access(BIN, os.X_OK)


@pytest.mark.gpu
def test_cpp_host_mirror_passes(cuda_dev):
    _build()
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "ALL PASSED" in r.stdout, r.stdout + r.stderr
