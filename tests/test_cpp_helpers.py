"""The C++ helper mirror (include/cbx_layer_helpers.hpp): it must compile and
link against libcbx_ops on the CPU box, and on a GPU its test program
(tests/cpp/test_layer_helpers.cpp) must pass against the oracle."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "test_layer_helpers.cpp")
CUDA = "/usr/local/cuda"


def _build(tmp_path):
    from chatterbox_amdvulkan_b200 import _lib, build
    import oracle
    if not os.path.exists(_lib.LIB_PATH):
        build.build()
    oracle.build()
    cxx = shutil.which("g++") or "/usr/bin/g++"
    exe = os.path.join(str(tmp_path), "test_layer_helpers")
    pkg, orc = os.path.dirname(_lib.LIB_PATH), os.path.dirname(oracle.LIB_PATH)
    cmd = [cxx, "-std=c++17", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), SRC, "-o", exe,
           "-L", pkg, "-lcbx_ops", "-L", orc, "-lcbx_oracle",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           f"-Wl,-rpath,{pkg}:{orc}:{os.path.join(CUDA, 'lib64')}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return exe


def test_cpp_helpers_compile_and_link(tmp_path):
    assert os.path.exists(_build(tmp_path))


@pytest.mark.gpu
def test_cpp_helpers_on_gpu(tmp_path):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASSED" in r.stdout
