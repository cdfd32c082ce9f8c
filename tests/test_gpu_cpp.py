"""The C++ host API (qwen3.8-27b-mlx_b200/cpp/gdn_delta.hpp) through a C++
port of the reference's test_delta (cpp/src/tests.cpp:196-243): the program
is compiled here against libgdn_b200.so and the C oracle, then run on the GPU."""
import os
import subprocess

import pytest

from conftest import PKG, ROOT

pytestmark = pytest.mark.gpu


def build_cpp_test(out):
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc"
    cmd = [nvcc, "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a", "-I", os.path.join(ROOT, "include"), "-I", os.path.join(PKG, "cpp"),
           os.path.join(ROOT, "tests", "cpp", "test_delta.cpp"), "-o", out,
           "-L", PKG, "-lgdn_b200", "-L", os.path.join(ROOT, "oracle"), "-loracle_gdn",
           "-Xlinker", f"-rpath={PKG}", "-Xlinker", f"-rpath={os.path.join(ROOT, 'oracle')}"]
    subprocess.run(cmd, check=True)


def test_cpp_delta_run_matches_oracle(tmp_path):
    exe = str(tmp_path / "test_delta")
    build_cpp_test(exe)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL PASS" in r.stdout
