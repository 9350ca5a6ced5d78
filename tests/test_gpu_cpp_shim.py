"""The C++ host shim (include/ks_evaluator.hpp) compiled into a small C++
program that calls the library like a reference C++ caller would."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpp_evaluator_shim(cuda_device, tmp_path):
    from comp390project_b200 import _capi
    lib = _capi.load()  # builds libks_b200.so if needed
    del lib
    libdir = os.path.dirname(_capi.lib_path())
    exe = str(tmp_path / "evaluator_selftest")
    subprocess.run(["nvcc", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "evaluator_selftest.cpp"), "-o", exe,
                    "-L", libdir, "-lks_b200", "-Xlinker", "-rpath=" + libdir], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "evaluator shim ok" in r.stdout
