"""The C++ host mirror (include/llmc_b200.hpp): it compiles and links against the library
here (no GPU needed), its host logic (tests/cpp/host_logic.cpp: target matching, the modifier
lifecycle, the session, the status mapping) passes on the CPU, and its known-answer test program
(tests/cpp/host_kats.cpp) passes on the GPU."""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _build(out_dir, name: str = "host_kats") -> str:
    from llmcompressorsharp_b200 import build

    lib = build.build()
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = os.path.join(str(out_dir), name)
    cmd = [gxx, "-std=c++17", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "cpp", name + ".cpp"), "-o", exe, "-L", os.path.dirname(lib), "-lllmc_b200",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", "-Wl,-rpath," + os.path.dirname(lib),
           "-Wl,-rpath," + os.path.join(CUDA, "lib64")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    return exe


def test_cpp_host_mirror_compiles_and_links(tmp_path):
    exe = _build(tmp_path)
    assert os.path.exists(exe)


def test_cpp_host_logic(tmp_path):
    exe = _build(tmp_path, "host_logic")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert " 0 failed" in r.stdout


@pytest.mark.gpu
def test_cpp_host_known_answers(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert " 0 failed" in r.stdout
