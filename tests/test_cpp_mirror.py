"""The C++ mirror of the forge-sort API (gpu-forge_b200/cpp/forge_sort.hpp):
compile tests/cpp/test_forge_sort.cpp against libforgesort.so and run it.
CPU: the tests that need no device (error strings, SortKey constants,
DeviceNotFound with every GPU hidden).  GPU: the whole suite."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "gpu-forge_b200", "forge_sort")


@pytest.fixture(scope="module")
def cpp_binary(tmp_path_factory):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    if not os.path.exists(os.path.join(LIBDIR, "libforgesort.so")):
        pytest.fail("libforgesort.so is not built (python gpu-forge_b200/build.py)")
    out = str(tmp_path_factory.mktemp("cpp") / "test_forge_sort")
    cmd = [cxx, "-std=c++20", "-O2", "-Wall", "-Wextra",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "gpu-forge_b200", "cpp"),
           os.path.join(ROOT, "tests", "cpp", "test_forge_sort.cpp"),
           "-L", LIBDIR, "-lforgesort", f"-Wl,-rpath,{LIBDIR}", "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    return out


def test_cpp_mirror_cpu(cpp_binary):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([cpp_binary, "--cpu"], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout


@pytest.mark.gpu
def test_cpp_mirror_gpu(cpp_binary):
    r = subprocess.run([cpp_binary], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "FAIL" not in r.stdout
